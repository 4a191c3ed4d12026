"""Parity at the benchmarked geometries, through the C ABI, against the oracle on the same inputs.

The small-geometry tests cover every code path; these cover the shapes the benchmark runs:

* Gemma-3-1B (d 1152, 26 layers, ff 6912): 36 and 216 blocks per row, so the exact int8 product runs
  its partial last K chunk on every projection, and 5 sliding layers per global one. 600 positions
  cross the 512-position window.
* Gemma-3-270M at the benchmark's own sequence (512 positions, seed 1000) through the default path:
  four parts on four streams, the third identical call replayed as a CUDA graph.
* The QAT layout (Q4_0 body, F16 output matrix) and the same model with the head requantized to
  Q8_0 at load (to_q8, crates/gem/src/q8.rs:129-145, called as model.rs:259-266).

Bar: argmax ids identical, log-probs within 1e-4 nats, tighter than the 1e-3 contract tolerance. The
forward and the logits are bit-identical; the log-probs differ only by the log-sum-exp summation order
over 2048 classes or 262144 rows, which over hundreds of positions reaches ~2.3e-5."""
import numpy as np
import pytest

from gem_b200 import FULL, TWO_LEVEL, Gemma, synth
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

LP_TOL = 1e-4
REF_THREADS = 8  # gem bench's pool size (crates/gem/src/main.rs:197)


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


def _check(g, o, toks, head, what):
    lp, am = g.score(toks, head)
    lpo, amo, _, _ = o.score(toks, head)
    err = float(np.abs(lp - lpo).max())
    assert err < LP_TOL, (what, head, err)
    assert np.array_equal(am, amo), (what, head, int(np.sum(am != amo)))
    return lp, am


@pytest.fixture(scope="module")
def m1b():
    return synth.ensure("gemma3-1b", classes=2048)  # shared cache with bench.py


@pytest.mark.parametrize("head,n", [(TWO_LEVEL, 600), (FULL, 64)])
def test_1b_geometry_exact(torch, isa, m1b, head, n):
    g = Gemma(m1b.gguf, ctx=1024)
    g.load_twolevel(m1b.twolevel)
    o = orc.Model(m1b.gguf, ctx=1024, threads=REF_THREADS, isa="avx512")
    o.load_twolevel(m1b.twolevel)
    _check(g, o, synth.tokens(n + 1, g.vocab, seed=3000), head, "1b")
    o.close()
    g.close()


@pytest.fixture(scope="module")
def m270():
    return synth.ensure("gemma3-270m", classes=2048)


def test_270m_bench_sequence_graph_replayed(torch, isa, m270):
    """bench.py's step: 512 positions of seed 1000, four parts, the third call a graph replay."""
    from gem_b200 import PARALLEL
    g = Gemma(m270.gguf, ctx=2048)
    g.load_twolevel(m270.twolevel)
    assert g.schedule_kind(TWO_LEVEL)[0] == PARALLEL
    o = orc.Model(m270.gguf, ctx=2048, threads=REF_THREADS, isa="avx512")
    o.load_twolevel(m270.twolevel)
    toks = synth.tokens(513, g.vocab, seed=1000)
    for head in (TWO_LEVEL, FULL):
        lpo, amo, _, _ = o.score(toks, head)
        for call in range(3):  # direct, captured, replayed
            lp, am = g.score(toks, head)
            assert np.abs(lp - lpo).max() < LP_TOL, (head, call, np.abs(lp - lpo).max())
            assert np.array_equal(am, amo), (head, call)
    o.close()
    g.close()


@pytest.fixture(scope="module")
def m270_qat():
    return synth.ensure("gemma3-270m", body="q4_0", head="f16", classes=2048)


@pytest.mark.parametrize("head_bits", [0, 8])
def test_270m_qat_layout(torch, isa, m270_qat, head_bits):
    """Q4_0 body with the F16 output matrix as stored (dot16) and requantized to Q8_0 at load."""
    g = Gemma(m270_qat.gguf, ctx=256, head_bits=head_bits)
    g.load_twolevel(m270_qat.twolevel)
    assert g.refresh_info()["head_bits"] == (16 if head_bits == 0 else 8)
    o = orc.Model(m270_qat.gguf, ctx=256, threads=REF_THREADS, isa="avx512", head_bits=head_bits)
    o.load_twolevel(m270_qat.twolevel)
    toks = synth.tokens(129, g.vocab, seed=4000 + head_bits)
    for head in (TWO_LEVEL, FULL):
        _check(g, o, toks, head, f"qat head_bits={head_bits}")
    o.close()
    g.close()


def test_f16_head_requantized_q8_small(torch, isa, tmp_path):
    """to_q8 of an F16 output matrix (f32 scales, round-half-away) at a ragged size: 1000 rows, 11
    blocks per row, under both heads and the per-token schedule too."""
    from gem_b200 import SEQUENTIAL
    cfg = dict(synth.SMALL, d=352, nh=4, nkv=1, hd=64, ff=512, vocab=1000, layers=2)
    path = synth.write_model(tmp_path / "f16head.gguf", cfg, seed=11, body="q4_0", head="f16")
    tl = synth.write_twolevel(tmp_path / "f16head-k8", cfg["vocab"], 8, cfg["d"], seed=12)
    o = orc.Model(path, ctx=128, threads=REF_THREADS, isa="avx512", head_bits=8)
    o.load_twolevel(tl)
    toks = synth.tokens(70, cfg["vocab"], seed=13)
    for schedule in (None, SEQUENTIAL):
        g = Gemma(path, ctx=128, head_bits=8)
        g.load_twolevel(tl)
        if schedule is not None:
            g.set_schedule(schedule)
        for head in (TWO_LEVEL, FULL):
            _check(g, o, toks, head, f"f16->q8 schedule={schedule}")
        g.close()
    o.close()


@pytest.mark.parametrize("head_bits", [0, 8, 4])
def test_twolevel_head_row_formats(torch, isa, tmp_path, head_bits):
    """The fused two-level head's block rows in every output-matrix format: F16 (dot16 on the fp32
    hidden state), Q8_0 and Q4_0 (requantized at load, f32 scales), through the per-token schedule and
    the batched entry point (batch 64: the class-logit product), against the oracle; 8 classes of 125 rows (the top class often differs
    from the target's, so both block paths run)."""
    from gem_b200 import SEQUENTIAL
    cfg = dict(synth.SMALL, d=352, nh=4, nkv=1, hd=64, ff=512, vocab=1000, layers=2)
    path = synth.write_model(tmp_path / "f16head.gguf", cfg, seed=11, body="q4_0", head="f16")
    tl = synth.write_twolevel(tmp_path / "f16head-k8", cfg["vocab"], 8, cfg["d"], seed=12)
    o = orc.Model(path, ctx=128, threads=REF_THREADS, isa="avx512", head_bits=head_bits)
    o.load_twolevel(tl)
    g = Gemma(path, ctx=128, head_bits=head_bits)
    g.load_twolevel(tl)
    g.set_schedule(SEQUENTIAL)
    _check(g, o, synth.tokens(40, cfg["vocab"], seed=14 + head_bits), TWO_LEVEL, f"two-level head_bits={head_bits}")
    rng = np.random.default_rng(15 + head_bits)
    for batch in (1, 5, 64):  # one round per CTA, two rounds (one launch), the class-logit product
        H = rng.standard_normal((batch, g.d)).astype(np.float32)
        Tg = rng.integers(0, g.vocab, batch).astype(np.uint32)
        Hd, Td = torch.tensor(H, device="cuda"), torch.tensor(Tg.astype(np.int32), device="cuda")
        lp = torch.empty(batch, device="cuda")
        am = torch.empty(batch, dtype=torch.int32, device="cuda")
        g.head_twolevel_dev(Hd.data_ptr(), Td.data_ptr(), batch, lp.data_ptr(), am.data_ptr())
        lp, am = lp.cpu().numpy(), am.cpu().numpy().astype(np.uint32)
        for b in range(batch):
            want_lp, want_am = o.twolevel(H[b], int(Tg[b]))
            assert abs(lp[b] - want_lp) < 2e-5 and am[b] == want_am, (batch, b, lp[b], want_lp, am[b], want_am)
    g.close()
    o.close()


@pytest.mark.parametrize("head_bits", [0, 8, 4])
def test_twolevel_head_large_classes(torch, isa, tmp_path, head_bits):
    """Classes of 300 rows: with the F16 output matrix the most likely class's block does not fit in
    shared memory at once (300 rows of 704 bytes), so the last CTA copies and scores it in two rounds;
    at batch 32 (one launch, 9 CTAs a hidden state) each CTA takes its 35 tasks in two rounds. The
    per-token schedule and the batched entry point at batch 1 and 32."""
    from gem_b200 import SEQUENTIAL
    cfg = dict(synth.SMALL, d=352, nh=4, nkv=1, hd=64, ff=512, vocab=2400, layers=2)
    path = synth.write_model(tmp_path / "bigclass.gguf", cfg, seed=21, body="q4_0", head="f16")
    tl = synth.write_twolevel(tmp_path / "bigclass-k8", cfg["vocab"], 8, cfg["d"], seed=22)
    o = orc.Model(path, ctx=128, threads=REF_THREADS, isa="avx512", head_bits=head_bits)
    o.load_twolevel(tl)
    g = Gemma(path, ctx=128, head_bits=head_bits)
    g.load_twolevel(tl)
    g.set_schedule(SEQUENTIAL)
    _check(g, o, synth.tokens(30, cfg["vocab"], seed=23 + head_bits), TWO_LEVEL, f"large classes head_bits={head_bits}")
    rng = np.random.default_rng(24 + head_bits)
    for batch in (1, 32):
        H = rng.standard_normal((batch, g.d)).astype(np.float32)
        Tg = rng.integers(0, g.vocab, batch).astype(np.uint32)
        Hd, Td = torch.tensor(H, device="cuda"), torch.tensor(Tg.astype(np.int32), device="cuda")
        lp = torch.empty(batch, device="cuda")
        am = torch.empty(batch, dtype=torch.int32, device="cuda")
        g.head_twolevel_dev(Hd.data_ptr(), Td.data_ptr(), batch, lp.data_ptr(), am.data_ptr())
        lp, am = lp.cpu().numpy(), am.cpu().numpy().astype(np.uint32)
        for b in range(batch):
            want_lp, want_am = o.twolevel(H[b], int(Tg[b]))
            assert abs(lp[b] - want_lp) < 2e-5 and am[b] == want_am, (batch, b, lp[b], want_lp, am[b], want_am)
    g.close()
    o.close()
