"""Batched scoring (independent sequences, each with its own KV slot) through the C ABI, checked
against the oracle scoring each sequence on its own: identical argmax ids, log-probs within the
log-sum-exp summation-order difference (2e-5, far inside the 1e-3 bar)."""
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


@pytest.fixture(scope="module")
def isa():
    if orc.detect_isa() != "avx512":
        pytest.skip("exact numerics reproduce the AVX-512 path; this host has none")


def _oracle_rows(path, twolevel, toks, head, ctx):
    o = orc.Model(path, ctx=ctx, threads=REF_THREADS, isa="avx512")
    o.load_twolevel(twolevel)
    out = [o.score(row, head)[:2] for row in toks]
    return np.stack([r[0] for r in out]), np.stack([r[1] for r in out])


@pytest.mark.parametrize("head", [FULL, TWO_LEVEL])
def test_batch_matches_oracle_with_regrouping(torch, isa, small, head):
    """5 sequences of 37 positions (a ragged last tile) on a model with 4 KV slots: two groups."""
    g = Gemma(small.gguf, ctx=128, max_seqs=4)
    g.load_twolevel(small.twolevel)
    toks = np.stack([synth.tokens(38, g.vocab, seed=200 + s) for s in range(5)])
    lp, am = g.score_batch(toks, head)
    lpo, amo = _oracle_rows(small.gguf, small.twolevel, toks, head, 128)
    assert np.abs(lp - lpo).max() < 2e-5, np.abs(lp - lpo).max()
    assert np.array_equal(am, amo)


def test_batch_equals_single_sequence_scoring(torch, small):
    g = Gemma(small.gguf, ctx=128, max_seqs=3)
    g.load_twolevel(small.twolevel)
    toks = np.stack([synth.tokens(50, g.vocab, seed=300 + s) for s in range(3)])
    lp, am = g.score_batch(toks, TWO_LEVEL)
    for s in range(3):
        l1, a1 = g.score(toks[s], TWO_LEVEL)
        assert np.array_equal(lp[s].view(np.uint32), l1.view(np.uint32)) and np.array_equal(am[s], a1)


def test_batch_long_sequences_chunked_by_position(torch, isa, small):
    """Two sequences longer than one chunk (1024 positions per sequence per chunk)."""
    g = Gemma(small.gguf, ctx=1200, max_seqs=2)
    g.load_twolevel(small.twolevel)
    toks = np.stack([synth.tokens(1101, g.vocab, seed=400 + s) for s in range(2)])
    lp, am = g.score_batch(toks, TWO_LEVEL)
    lpo, amo = _oracle_rows(small.gguf, small.twolevel, toks, TWO_LEVEL, 1200)
    assert np.abs(lp - lpo).max() < 2e-5 and np.array_equal(am, amo)


def test_batch_device_buffers(torch, small):
    g = Gemma(small.gguf, ctx=128, max_seqs=8)
    g.load_twolevel(small.twolevel)
    toks = np.stack([synth.tokens(33, g.vocab, seed=500 + s) for s in range(6)])
    want, want_am = g.score_batch(toks, TWO_LEVEL)
    td = torch.tensor(toks.astype(np.int32), device="cuda")
    lp = torch.empty((6, 32), device="cuda")
    am = torch.empty((6, 32), dtype=torch.int32, device="cuda")
    g.score_batch_dev(td.data_ptr(), 6, 32, TWO_LEVEL, lp.data_ptr(), am.data_ptr())
    g.sync()
    assert np.array_equal(lp.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert np.array_equal(am.cpu().numpy().astype(np.uint32), want_am)


def test_batch_with_bos_model(torch, isa, model_dir):
    """A model whose tokenizer adds BOS: every sequence starts with the same BOS forward."""
    cfg = synth.CONFIGS["small"]
    path = synth.write_model(model_dir / "small-bos.gguf", cfg, seed=11, bos=True)
    prefix = synth.write_twolevel(model_dir / "small-bos", cfg["vocab"], 64, cfg["d"], seed=11)
    g = Gemma(path, ctx=128, max_seqs=2)
    g.load_twolevel(prefix)
    assert g.bos >= 0
    toks = np.stack([synth.tokens(30, g.vocab, seed=600 + s) for s in range(3)])
    lp, am = g.score_batch(toks, TWO_LEVEL)
    lpo, amo = _oracle_rows(path, prefix, toks, TWO_LEVEL, 128)
    assert np.abs(lp - lpo).max() < 2e-5 and np.array_equal(am, amo)
