"""Checks against the committed fixtures in tests/golden (written by tests/golden/make_golden.py).

gem has no test vectors of its own. The fixtures hold what two independent implementations compute
on the seeded synthetic models (gguf-py's block dequantization; transformers' Gemma 3 and Qwen2
forwards) and the oracle's AVX-512 outputs, frozen. On the CPU: the synthetic models are regenerated
byte for byte, and the oracle reproduces its frozen outputs exactly and stays within the int8
activation noise of transformers. On the GPU (through the C ABI): every schedule reproduces the frozen
hidden states bit for bit and the log-probs and argmax ids, with no need for an AVX-512 host."""
import hashlib
from pathlib import Path

import numpy as np
import pytest

from gem_b200 import FULL, TWO_LEVEL, synth
from oracle import oracle as orc

GOLDEN = Path(__file__).resolve().parent / "golden"
MODELS = {"small": "small_gemma3.npz", "small-qwen2": "small_qwen2.npz"}
REF_THREADS = 8
LP_TOL = 1e-3     # per-token log-prob tolerance (absolute, nats)


def _fixture(name):
    return np.load(GOLDEN / MODELS[name])


def _sha256(*paths):
    h = hashlib.sha256()
    for p in paths:
        h.update(Path(p).read_bytes())
    return h.hexdigest()


@pytest.fixture(scope="module", params=list(MODELS))
def golden(request, model_dir):
    files = synth.ensure(request.param, classes=64, directory=model_dir)
    return request.param, files, _fixture(request.param)


@pytest.mark.parametrize("qtype,kind", [("Q8_0", 8), ("Q4_0", 2)])
def test_block_dequant_matches_gguf_py_golden(qtype, kind):
    fx = np.load(GOLDEN / "gguf_blocks.npz")
    rows, cols = fx["w"].shape
    got = orc.Mat(kind, fx[f"{qtype}_raw"], rows, cols).dequant()
    assert np.array_equal(got.view(np.uint32), fx[f"{qtype}_dequant"].view(np.uint32))


def test_synthetic_models_are_the_golden_ones(golden):
    name, files, fx = golden
    assert _sha256(files.gguf) == str(fx["gguf_sha256"]), f"{name}: regenerate tests/golden (synth changed)"
    p = str(files.twolevel)
    assert _sha256(p + ".order", p + ".A", p + ".b") == str(fx["twolevel_sha256"])


def test_oracle_within_activation_noise_of_transformers_golden(golden, threads):
    name, files, fx = golden
    o = orc.Model(files.gguf, ctx=128, threads=threads)
    lp, _, _, _ = o.score(fx["hf_tokens"], FULL)
    d = np.abs(lp - fx["hf_lp"])
    # int8 activation quantization (Act::quantize) against transformers' fp32 activations
    assert d.max() < 0.05 and d.mean() < 0.015, (name, d.max(), d.mean())


def test_oracle_reproduces_frozen_outputs(golden):
    name, files, fx = golden
    if orc.detect_isa() != "avx512":
        pytest.skip("the frozen outputs are the AVX-512 path's; this host has none")
    o = orc.Model(files.gguf, ctx=128, threads=REF_THREADS, isa="avx512")
    o.load_twolevel(files.twolevel)
    for tag, head in (("full", FULL), ("twolevel", TWO_LEVEL)):
        lp, am, _, _ = o.score(fx["tokens"], head)
        assert np.array_equal(lp.view(np.uint32), fx[f"lp_{tag}"].view(np.uint32)), (name, tag)
        assert np.array_equal(am, fx[f"am_{tag}"]), (name, tag)
    o = orc.Model(files.gguf, ctx=128, threads=REF_THREADS, isa="avx512")
    want = dict(zip(fx["hidden_pos"].tolist(), fx["hidden"]))
    for i, t in enumerate(fx["tokens"][:max(want) + 1]):
        h = o.forward(int(t), i)
        if i in want:
            assert np.array_equal(h.view(np.uint32), want[i].view(np.uint32)), (name, i)


@pytest.mark.gpu
@pytest.mark.parametrize("schedule", ["sequential", "pipelined", "parallel"])
def test_gpu_scores_match_golden(golden, schedule):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gem_b200 import PARALLEL, PIPELINED, SEQUENTIAL, Gemma
    name, files, fx = golden
    g = Gemma(files.gguf, ctx=128)
    g.load_twolevel(files.twolevel)
    g.set_schedule({"sequential": SEQUENTIAL, "pipelined": PIPELINED, "parallel": PARALLEL}[schedule])
    for tag, head in (("full", FULL), ("twolevel", TWO_LEVEL)):
        lp, am = g.score(fx["tokens"], head)
        assert np.abs(lp - fx[f"lp_{tag}"]).max() < LP_TOL
        assert np.abs(lp - fx[f"lp_{tag}"]).max() < 2e-5, (name, tag)  # only the log-sum-exp order differs
        assert np.array_equal(am, fx[f"am_{tag}"]), (name, tag)


@pytest.mark.gpu
def test_gpu_hidden_states_match_golden(golden):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gem_b200 import Gemma
    name, files, fx = golden
    g = Gemma(files.gguf, ctx=128)
    want = dict(zip(fx["hidden_pos"].tolist(), fx["hidden"]))
    for i, t in enumerate(fx["tokens"][:max(want) + 1]):
        h = g.forward(int(t), i)
        if i in want:
            assert np.array_equal(h.view(np.uint32), want[i].view(np.uint32)), (name, i)
