"""Generation-side heads through the C ABI against the oracle: greedy screening (lean.rs:46-107),
two-level sampling (main.rs:109-141) and the completion loop, on the small model with exact numerics:
identical tokens (and identical generator state after sampling)."""
import numpy as np
import pytest

from gem_b200 import GREEDY_FULL, GREEDY_SCREEN, SAMPLE, Gemma, synth
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


def _models(small, ctx=256):
    g = Gemma(small.gguf, ctx=ctx)
    g.load_twolevel(small.twolevel)
    o = orc.Model(small.gguf, ctx=ctx, threads=REF_THREADS, isa="avx512")
    o.load_twolevel(small.twolevel)
    return g, o


def _median_gap(small, H):
    """A confidence floor halfway between two consecutive items' top-class probabilities (float64),
    so that about half the items fall back and none sits near the threshold."""
    A = np.fromfile(str(small.twolevel) + ".A", dtype="<f4").reshape(-1, H.shape[1]).astype(np.float64)
    b = np.fromfile(str(small.twolevel) + ".b", dtype="<f4").astype(np.float64)
    cl = H.astype(np.float64) @ A.T + b
    p = np.sort(np.exp(cl.max(1) - (cl.max(1) + np.log(np.exp(cl - cl.max(1, keepdims=True)).sum(1)))))
    i = len(p) // 2
    return float((p[i - 1] + p[i]) / 2)


@pytest.mark.parametrize("top,always,min_conf", [(1, (), 0.0), (3, (), 0.0), (2, (5, 700, 8000), 0.0), (1, (), None)])
def test_greedy_screening_matches_oracle(torch, isa, small, top, always, min_conf):
    g, o = _models(small)
    rng = np.random.default_rng(7 + top)
    H = (rng.standard_normal((24, g.d)) * 2).astype(np.float32)
    if min_conf is None:
        min_conf = _median_gap(small, H)
    Hd = torch.tensor(H, device="cuda")
    al = torch.tensor(np.asarray(always, np.int32) if always else np.zeros(1, np.int32), device="cuda")
    tok = torch.empty(24, dtype=torch.int32, device="cuda")
    fb = torch.empty(24, dtype=torch.int32, device="cuda")
    g.greedy_dev(Hd.data_ptr(), 24, top, min_conf, al.data_ptr(), len(always), tok.data_ptr(), fb.data_ptr())
    g.sync()
    tok, fb = tok.cpu().numpy().astype(np.uint32), fb.cpu().numpy()
    fell = 0
    for i in range(24):
        want, wfb = o.greedy(H[i], top, min_conf, always)
        assert tok[i] == want, (i, tok[i], want)
        if min_conf > 0:
            assert bool(fb[i]) == wfb
            fell += wfb
    if min_conf > 0:
        assert 0 < fell < 24  # both paths exercised


def test_sampling_matches_oracle(torch, isa, small):
    g, o = _models(small)
    toks = synth.tokens(12, g.vocab, seed=41)
    for i, t in enumerate(toks):
        g.forward(int(t), i)
        h = o.forward(int(t), i)
    r1 = r2 = 0x9E3779B97F4A7C15
    for _ in range(40):
        a, r1 = g.sample(0.8, r1)
        b, r2 = o.sample(h, 0.8, r2)
        assert a == b and r1 == r2


@pytest.mark.parametrize("mode", [GREEDY_FULL, GREEDY_SCREEN, SAMPLE])
def test_generate_matches_oracle_loop(torch, isa, small, mode):
    g, o = _models(small)
    prompt = synth.tokens(9, g.vocab, seed=50 + mode)
    kw = dict(top=2, always=(3, 4000), temperature=0.7, seed=12345)
    got = g.generate(prompt, 20, mode=mode, **kw)
    for i, t in enumerate(prompt):  # the oracle's loop (lean.rs:180-200)
        h = o.forward(int(t), i)
    pos, rng, want = len(prompt), kw["seed"], []
    for _ in range(20):
        if mode == GREEDY_FULL:
            t = o.full(h, 0)[1]
        elif mode == GREEDY_SCREEN:
            t = o.greedy(h, kw["top"], 0.0, kw["always"])[0]
        else:
            t, rng = o.sample(h, kw["temperature"], rng)
        want.append(t)
        h = o.forward(int(t), pos)
        pos += 1
    assert list(got) == want


def test_generate_stops(torch, small):
    g, _ = _models(small)
    prompt = synth.tokens(5, g.vocab, seed=60)
    free = g.generate(prompt, 12, mode=GREEDY_FULL)
    stopped = g.generate(prompt, 12, mode=GREEDY_FULL, stops=(int(free[4]),))
    assert list(stopped) == list(free[:list(free).index(free[4])])
