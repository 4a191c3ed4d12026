"""The parallel schedule's body products on the tensor cores (gem_set_tensor_cores, tc_gemm.cu).

The tensor cores form each lane's exact int8 pair sums and the CUDA cores apply the reference's one
fp32 FMA per lane and block (crates/gem/src/q8.rs:257-270), so scoring with them on must give results
bit-identical to the CUDA-core products, and so to the oracle's AVX-512 path: same log-probs bit for
bit, same argmax ids. Covered: both heads, a sequence in four parts (512 positions: ragged last tile of
12 positions), a short ragged chunk, the Q4_0 body, f32 scales after requantization, batched scoring,
and the 270M geometry on the benchmark's own sequence."""
import numpy as np
import pytest

from gem_b200 import FULL, TWO_LEVEL, Gemma, synth
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

REF_THREADS = 8


@pytest.fixture(scope="module")
def torch():
    import torch as t
    if not t.cuda.is_available():
        pytest.skip("no CUDA device")
    return t


def _pair(path, twolevel, **kw):
    a = Gemma(path, **kw)
    b = Gemma(path, **kw)
    for g in (a, b):
        g.load_twolevel(twolevel)
    b.set_tensor_cores(True)
    return a, b


def _same(x, y):
    return np.array_equal(x[0].view(np.uint32), y[0].view(np.uint32)) and np.array_equal(x[1], y[1])


@pytest.mark.parametrize("n", [20, 512])
@pytest.mark.parametrize("body_bits,head_bits", [(8, 0), (4, 0), (8, 8)])
def test_tensor_core_products_are_bit_identical(torch, small, n, body_bits, head_bits):
    cuda, tc = _pair(small.gguf, small.twolevel, ctx=600, body_bits=body_bits, head_bits=head_bits)
    toks = synth.tokens(n + 1, small.cfg["vocab"], seed=500 + n)
    for head in (FULL, TWO_LEVEL):
        for call in range(3):  # direct, captured as a graph, replayed
            assert _same(cuda.score(toks, head), tc.score(toks, head)), (head, call)
    cuda.close()
    tc.close()


def test_tensor_core_batched_scoring(torch, small):
    cuda, tc = _pair(small.gguf, small.twolevel, ctx=128, max_seqs=4)
    toks = np.stack([synth.tokens(70, small.cfg["vocab"], seed=600 + s) for s in range(6)])
    for head in (FULL, TWO_LEVEL):
        assert _same(cuda.score_batch(toks, head), tc.score_batch(toks, head)), head
    cuda.close()
    tc.close()


def test_tensor_core_270m_bench_sequence_against_oracle(torch):
    if orc.detect_isa() != "avx512":
        pytest.skip("exact numerics reproduce the AVX-512 path; this host has none")
    m = synth.ensure("gemma3-270m", classes=2048)
    g = Gemma(m.gguf, ctx=2048)
    g.load_twolevel(m.twolevel)
    g.set_tensor_cores(True)
    o = orc.Model(m.gguf, ctx=2048, threads=REF_THREADS, isa="avx512")
    o.load_twolevel(m.twolevel)
    toks = synth.tokens(513, g.vocab, seed=1000)
    lp, am = g.score(toks, TWO_LEVEL)
    lpo, amo, _, _ = o.score(toks, TWO_LEVEL)
    assert np.abs(lp - lpo).max() < 1e-4 and np.array_equal(am, amo)
    o.close()
    g.close()
