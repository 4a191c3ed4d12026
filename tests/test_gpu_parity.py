"""Parity of the sm_100a path (through the C ABI) with the oracle on identical seeded inputs.

Bars: identical argmax token ids, per-token log-probs within 1e-3 absolute,
dequantized weights bit-exact. Kernel-level GEMV outputs agree to fp32 summation-order noise."""
import numpy as np
import pytest

from gem_b200 import FULL, TWO_LEVEL, Gemma, synth
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

LP_TOL = 1e-3


@pytest.fixture(scope="module")
def torch():
    import torch as t
    if not t.cuda.is_available():
        pytest.skip("no CUDA device")
    return t


def _gguf_mat(path, name):
    import gguf
    r = gguf.GGUFReader(str(path))
    t = next(t for t in r.tensors if t.name == name)
    kind = {gguf.GGMLQuantizationType.Q8_0: 8, gguf.GGMLQuantizationType.Q4_0: 2, gguf.GGMLQuantizationType.F16: 1}[t.tensor_type]
    rows, cols = int(t.shape[1]), int(t.shape[0])
    return orc.Mat(kind, np.ascontiguousarray(t.data).view(np.uint8).reshape(-1), rows, cols)


NAMES = ["attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"]


@pytest.mark.parametrize("which", range(7))
def test_matvec_matches_oracle(torch, small, which):
    g = Gemma(small.gguf, ctx=64)
    m = _gguf_mat(small.gguf, f"blk.1.{NAMES[which]}.weight")
    rng = np.random.default_rng(20 + which)
    x = rng.standard_normal(m.cols).astype(np.float32)
    xd = torch.tensor(x, device="cuda")
    yd = torch.empty(m.rows, device="cuda")
    g.matvec_dev(1, which, xd.data_ptr(), yd.data_ptr())
    want = m.matvec(x, "avx2", threads=1)
    np.testing.assert_allclose(yd.cpu().numpy(), want, rtol=1e-5, atol=1e-6)


def test_head_matvec_matches_oracle(torch, small):
    g = Gemma(small.gguf, ctx=64)
    m = _gguf_mat(small.gguf, "token_embd.weight")
    x = np.random.default_rng(30).standard_normal(m.cols).astype(np.float32)
    xd = torch.tensor(x, device="cuda")
    yd = torch.empty(m.rows, device="cuda")
    g.matvec_dev(-1, 0, xd.data_ptr(), yd.data_ptr())
    np.testing.assert_allclose(yd.cpu().numpy(), m.matvec(x, "avx2", threads=4), rtol=1e-5, atol=1e-6)


def test_forward_hidden_state_tracks_oracle(torch, small, threads):
    g = Gemma(small.gguf, ctx=128)
    o = orc.Model(small.gguf, ctx=128, threads=threads)
    toks = synth.tokens(40, g.vocab, seed=3)
    worst = 0.0
    for i, t in enumerate(toks):
        hg = g.forward(int(t), i)
        ho = o.forward(int(t), i)
        worst = max(worst, float(np.abs(hg - ho).max()))
        assert np.abs(hg - ho).mean() < 1e-3, (i, np.abs(hg - ho).mean())
    assert worst < 5e-2


@pytest.mark.parametrize("head", [FULL, TWO_LEVEL])
def test_score_matches_oracle(torch, small, threads, head):
    g = Gemma(small.gguf, ctx=128)
    g.load_twolevel(small.twolevel)
    o = orc.Model(small.gguf, ctx=128, threads=threads)
    o.load_twolevel(small.twolevel)
    toks = synth.tokens(49, g.vocab, seed=5)
    lp, am = g.score(toks, head)
    lpo, amo, _, _ = o.score(toks, head)
    assert np.abs(lp - lpo).max() < LP_TOL, np.abs(lp - lpo).max()
    assert np.array_equal(am, amo)


@pytest.mark.parametrize("batch", [1, 64])
def test_head_batch_matches_oracle(torch, small, threads, batch):
    g = Gemma(small.gguf, ctx=64)
    g.load_twolevel(small.twolevel)
    o = orc.Model(small.gguf, ctx=64, threads=threads)
    o.load_twolevel(small.twolevel)
    rng = np.random.default_rng(40 + batch)
    H = rng.standard_normal((batch, g.d)).astype(np.float32)
    T = rng.integers(0, g.vocab, batch).astype(np.uint32)
    Hd, Td = torch.tensor(H, device="cuda"), torch.tensor(T.astype(np.int32), device="cuda")
    for which, fn in ((FULL, g.head_full_dev), (TWO_LEVEL, g.head_twolevel_dev)):
        lp = torch.empty(batch, device="cuda")
        am = torch.empty(batch, dtype=torch.int32, device="cuda")
        fn(Hd.data_ptr(), Td.data_ptr(), batch, lp.data_ptr(), am.data_ptr())
        lp, am = lp.cpu().numpy(), am.cpu().numpy().astype(np.uint32)
        for b in range(batch):
            want = o.full(H[b], int(T[b])) if which == FULL else o.twolevel(H[b], int(T[b]))
            assert abs(lp[b] - want[0]) < LP_TOL, (which, b, lp[b], want[0])
            assert am[b] == want[1], (which, b)
