"""Parity of the sm_100a path (through the C ABI) with the oracle on identical seeded inputs.

Exact numerics (the default): hidden states and logits bit-identical to the oracle's AVX-512 path
with the same pool size; log-probs within 1e-3 (they differ only in log-sum-exp summation order, so in
practice ~1e-6); argmax token ids identical; dequantized weights bit-exact.

Fast numerics: tree reductions make int8 quantization flips diverge from the oracle the same way the
reference's own AVX2 and AVX-512 paths diverge from each other, so the bar is that spread."""
import numpy as np
import pytest

from gem_b200 import EXACT, FAST, FULL, TWO_LEVEL, Gemma, synth
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

LP_TOL = 1e-3      # per-token log-prob tolerance of the contract (absolute, nats)
REF_THREADS = 8    # gem bench's default pool size (crates/gem/src/main.rs:197)


@pytest.fixture(scope="module")
def torch():
    import torch as t
    if not t.cuda.is_available():
        pytest.skip("no CUDA device")
    return t


@pytest.fixture(scope="module")
def isa():
    i = orc.detect_isa()
    if i != "avx512":
        pytest.skip("exact numerics reproduce the AVX-512 path; this host has none")
    return i


def _gguf_mat(path, name):
    import gguf
    r = gguf.GGUFReader(str(path))
    t = next(t for t in r.tensors if t.name == name)
    kind = {gguf.GGMLQuantizationType.Q8_0: 8, gguf.GGMLQuantizationType.Q4_0: 2, gguf.GGMLQuantizationType.F16: 1}[t.tensor_type]
    rows, cols = int(t.shape[1]), int(t.shape[0])
    return orc.Mat(kind, np.ascontiguousarray(t.data).view(np.uint8).reshape(-1), rows, cols)


NAMES = ["attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"]


@pytest.mark.parametrize("which", range(7))
def test_matvec_bit_exact(torch, isa, small, which):
    g = Gemma(small.gguf, ctx=64)
    m = _gguf_mat(small.gguf, f"blk.1.{NAMES[which]}.weight")
    x = np.random.default_rng(20 + which).standard_normal(m.cols).astype(np.float32)
    xd = torch.tensor(x, device="cuda")
    yd = torch.empty(m.rows, device="cuda")
    g.matvec_dev(1, which, xd.data_ptr(), yd.data_ptr())
    want = m.matvec(x, "avx512", threads=1)
    assert np.array_equal(yd.cpu().numpy().view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("which", [0, 6])
def test_matvec_fast_close(torch, small, which):
    g = Gemma(small.gguf, ctx=64)
    g.set_numerics(FAST)
    m = _gguf_mat(small.gguf, f"blk.2.{NAMES[which]}.weight")
    x = np.random.default_rng(50 + which).standard_normal(m.cols).astype(np.float32)
    xd = torch.tensor(x, device="cuda")
    yd = torch.empty(m.rows, device="cuda")
    g.matvec_dev(2, which, xd.data_ptr(), yd.data_ptr())
    np.testing.assert_allclose(yd.cpu().numpy(), m.matvec(x, "avx2", threads=1), rtol=1e-5, atol=1e-6)


def test_head_matvec_bit_exact(torch, isa, small):
    g = Gemma(small.gguf, ctx=64)
    m = _gguf_mat(small.gguf, "token_embd.weight")
    x = np.random.default_rng(30).standard_normal(m.cols).astype(np.float32)
    xd = torch.tensor(x, device="cuda")
    yd = torch.empty(m.rows, device="cuda")
    g.matvec_dev(-1, 0, xd.data_ptr(), yd.data_ptr())
    assert np.array_equal(yd.cpu().numpy().view(np.uint32), m.matvec(x, "avx512", threads=4).view(np.uint32))


def test_forward_hidden_state_bit_exact(torch, isa, small):
    g = Gemma(small.gguf, ctx=128)
    o = orc.Model(small.gguf, ctx=128, threads=REF_THREADS, isa="avx512")
    toks = synth.tokens(40, g.vocab, seed=3)
    for i, t in enumerate(toks):  # 40 positions: past the 16-token window, through the global layer
        hg = g.forward(int(t), i)
        ho = o.forward(int(t), i)
        assert np.array_equal(hg.view(np.uint32), ho.view(np.uint32)), (i, np.abs(hg - ho).max())


@pytest.mark.parametrize("schedule", ["sequential", "pipelined", "parallel"])
@pytest.mark.parametrize("head", [FULL, TWO_LEVEL])
def test_score_exact(torch, isa, small, head, schedule):
    from gem_b200 import PARALLEL, PIPELINED, SEQUENTIAL
    g = Gemma(small.gguf, ctx=128)
    g.load_twolevel(small.twolevel)
    g.set_schedule({"sequential": SEQUENTIAL, "pipelined": PIPELINED, "parallel": PARALLEL}[schedule])
    o = orc.Model(small.gguf, ctx=128, threads=REF_THREADS, isa="avx512")
    o.load_twolevel(small.twolevel)
    toks = synth.tokens(49, g.vocab, seed=5)
    lp, am = g.score(toks, head)
    lpo, amo, _, _ = o.score(toks, head)
    assert np.abs(lp - lpo).max() < LP_TOL
    assert np.abs(lp - lpo).max() < 2e-5  # only the log-sum-exp order differs
    assert np.array_equal(am, amo)


@pytest.mark.parametrize("batch", [1, 64])
def test_head_batch_exact(torch, isa, small, threads, batch):
    g = Gemma(small.gguf, ctx=64)
    g.load_twolevel(small.twolevel)
    o = orc.Model(small.gguf, ctx=64, threads=threads, isa="avx512")
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
            assert abs(lp[b] - want[0]) < 2e-5, (which, b, lp[b], want[0])
            assert am[b] == want[1], (which, b)


@pytest.mark.parametrize("head", [FULL, TWO_LEVEL])
def test_score_fast_within_reference_isa_spread(torch, isa, small, head):
    from gem_b200 import SEQUENTIAL
    g = Gemma(small.gguf, ctx=128)
    g.set_numerics(FAST)
    g.set_schedule(SEQUENTIAL)  # the parallel schedule always computes exactly
    g.load_twolevel(small.twolevel)
    toks = synth.tokens(49, g.vocab, seed=6)
    lp, am = g.score(toks, head)
    ref = {}
    for i in ("avx512", "avx2"):
        o = orc.Model(small.gguf, ctx=128, threads=REF_THREADS, isa=i)
        o.load_twolevel(small.twolevel)
        ref[i] = o.score(toks, head)[:2]
    spread = np.abs(ref["avx512"][0] - ref["avx2"][0])
    ours = np.abs(lp - ref["avx512"][0])
    # The reference's own AVX-512 / AVX2 / scalar paths differ by up to ~0.045 nats per token on the
    # 270M geometry (mean ~0.01): fast numerics must stay in that band.
    assert ours.max() <= 0.05
    assert ours.mean() <= 3 * max(spread.mean(), 1e-3)
    assert (am == ref["avx512"][1]).mean() >= 0.9


def test_pipelined_and_sequential_schedules_agree(torch, isa, small):
    from gem_b200 import PIPELINED, SEQUENTIAL
    g = Gemma(small.gguf, ctx=128)
    g.load_twolevel(small.twolevel)
    g.set_schedule(PIPELINED)
    pipelined, G, GH, why = g.schedule(TWO_LEVEL)
    assert pipelined, why
    toks = synth.tokens(60, g.vocab, seed=12)
    lp_p, am_p = g.score(toks, TWO_LEVEL)
    g.set_schedule(SEQUENTIAL)
    assert not g.schedule(TWO_LEVEL)[0]
    lp_s, am_s = g.score(toks, TWO_LEVEL)
    assert np.abs(lp_p - lp_s).max() < 2e-5 and np.array_equal(am_p, am_s)
    o = orc.Model(small.gguf, ctx=128, threads=REF_THREADS, isa="avx512")
    o.load_twolevel(small.twolevel)
    lpo, amo, _, _ = o.score(toks, TWO_LEVEL)
    assert np.abs(lp_p - lpo).max() < 2e-5 and np.array_equal(am_p, amo)
    # the pipelined kernel also leaves the last hidden state for single-token head calls
    g.set_schedule(PIPELINED)
    g.score(toks, TWO_LEVEL)
    lp1, am1 = g.twolevel_logprob(int(toks[-1]))
    assert abs(lp1 - lp_p[-1]) < 2e-5 and am1 == am_p[-1]


def test_pipeline_bounded_wait_reports_timeout(torch, small):
    from gem_b200 import PIPELINED, GemError
    g = Gemma(small.gguf, ctx=64)
    g.load_twolevel(small.twolevel)
    g.set_schedule(PIPELINED)
    toks = synth.tokens(20, g.vocab, seed=13)
    want, _ = g.score(toks, TWO_LEVEL)
    g.test_withhold_stage(2, wait_ms=200)
    with pytest.raises(GemError) as e:
        g.score(toks, TWO_LEVEL)
    assert e.value.code == -9  # GEM_E_TIMEOUT
    g.test_withhold_stage(-1, wait_ms=2000)
    g.reset(0)
    again, _ = g.score(toks, TWO_LEVEL)  # the context is still usable
    assert np.abs(again - want).max() < 2e-5


@pytest.fixture(scope="module")
def m270():
    return synth.ensure("gemma3-270m", classes=2048)  # shared cache with bench.py


@pytest.mark.parametrize("schedule", ["pipelined", "parallel"])
def test_270m_scoring_is_exact(torch, isa, m270, schedule):
    from gem_b200 import PARALLEL, PIPELINED
    g = Gemma(m270.gguf, ctx=2048)
    g.load_twolevel(m270.twolevel)
    g.set_schedule(PIPELINED if schedule == "pipelined" else PARALLEL)
    assert g.schedule_kind(TWO_LEVEL)[0] == (PIPELINED if schedule == "pipelined" else PARALLEL)
    o = orc.Model(m270.gguf, ctx=2048, threads=REF_THREADS, isa="avx512")
    o.load_twolevel(m270.twolevel)
    toks = synth.tokens(97, g.vocab, seed=21)
    lp, am = g.score(toks, TWO_LEVEL)
    lpo, amo, _, _ = o.score(toks, TWO_LEVEL)
    assert np.abs(lp - lpo).max() < 2e-5, np.abs(lp - lpo).max()
    assert np.array_equal(am, amo)
    lpf, amf = g.score(toks, FULL)
    lpfo, amfo, _, _ = o.score(toks, FULL)
    assert np.abs(lpf - lpfo).max() < 1e-4 and np.array_equal(amf, amfo)


def test_parallel_schedule_is_auto_default(torch, small):
    from gem_b200 import PARALLEL
    g = Gemma(small.gguf, ctx=64)
    g.load_twolevel(small.twolevel)
    assert g.schedule_kind(TWO_LEVEL)[0] == PARALLEL and g.schedule_kind(FULL)[0] == PARALLEL


@pytest.mark.parametrize("n", [1, 33, 1100])
def test_parallel_lengths_and_chunks(torch, isa, small, n):
    """A single position, a ragged tile (33 = 32 + 1) and two chunks (1100 > 1024 positions per chunk,
    the second chunk's attention reading K/V rows the first chunk wrote)."""
    g = Gemma(small.gguf, ctx=1200)
    g.load_twolevel(small.twolevel)
    o = orc.Model(small.gguf, ctx=1200, threads=REF_THREADS, isa="avx512")
    o.load_twolevel(small.twolevel)
    toks = synth.tokens(n + 1, g.vocab, seed=70 + n)
    lp, am = g.score(toks, TWO_LEVEL)
    lpo, amo, _, _ = o.score(toks, TWO_LEVEL)
    assert np.abs(lp - lpo).max() < 2e-5 and np.array_equal(am, amo)
    # the last position's hidden state is left for single-token head calls
    lp1, am1 = g.twolevel_logprob(int(toks[-1]))
    assert abs(lp1 - lp[-1]) < 2e-5 and am1 == am[-1]


@pytest.mark.parametrize("body_bits,head_bits", [(4, 0), (8, 4), (4, 8)])
def test_parallel_requantized_formats(torch, isa, small, body_bits, head_bits):
    """--body-bits / --head-bits (to_q4 / to_q8, q8.rs:129-165; f32 scales) through the exact GEMM."""
    g = Gemma(small.gguf, ctx=128, body_bits=body_bits, head_bits=head_bits)
    g.load_twolevel(small.twolevel)
    o = orc.Model(small.gguf, ctx=128, threads=REF_THREADS, isa="avx512", body_bits=body_bits, head_bits=head_bits)
    o.load_twolevel(small.twolevel)
    toks = synth.tokens(41, g.vocab, seed=90 + body_bits + head_bits)
    for head in (FULL, TWO_LEVEL):
        lp, am = g.score(toks, head)
        lpo, amo, _, _ = o.score(toks, head)
        assert np.abs(lp - lpo).max() < 2e-5 and np.array_equal(am, amo), (head, np.abs(lp - lpo).max())


@pytest.fixture(scope="module")
def small_qwen2(model_dir):
    return synth.ensure("small-qwen2", classes=64, directory=model_dir)


@pytest.mark.parametrize("schedule", ["sequential", "parallel"])
@pytest.mark.parametrize("head", [FULL, TWO_LEVEL])
def test_qwen2_scoring_exact(torch, isa, small_qwen2, head, schedule):
    """The qwen2 branch (biases, SiLU, untied output, 7 query heads per kv head) under both schedules."""
    from gem_b200 import PARALLEL, SEQUENTIAL
    g = Gemma(small_qwen2.gguf, ctx=128)
    g.load_twolevel(small_qwen2.twolevel)
    g.set_schedule(SEQUENTIAL if schedule == "sequential" else PARALLEL)
    o = orc.Model(small_qwen2.gguf, ctx=128, threads=REF_THREADS, isa="avx512")
    o.load_twolevel(small_qwen2.twolevel)
    toks = synth.tokens(45, g.vocab, seed=77)
    lp, am = g.score(toks, head)
    lpo, amo, _, _ = o.score(toks, head)
    assert np.abs(lp - lpo).max() < 2e-5 and np.array_equal(am, amo), np.abs(lp - lpo).max()


def test_qwen2_forward_bit_exact(torch, isa, small_qwen2):
    g = Gemma(small_qwen2.gguf, ctx=64)
    o = orc.Model(small_qwen2.gguf, ctx=64, threads=REF_THREADS, isa="avx512")
    for i, t in enumerate(synth.tokens(20, g.vocab, seed=78)):
        assert np.array_equal(g.forward(int(t), i).view(np.uint32), o.forward(int(t), i).view(np.uint32)), i


@pytest.mark.parametrize("batch", [1, 3, 13])
def test_head_full_partial_row_groups(torch, isa, threads, tmp_path, batch):
    """An output matrix whose rows fill neither 16-row groups nor 8-group stages (1000 rows): the
    streamed full head (batches below 12) reads a short last stage and a half-filled last group, the
    matrix-product path (12 and more) a partial row tile; both against the oracle."""
    cfg = dict(synth.SMALL, vocab=1000, layers=1)
    path = synth.write_model(tmp_path / "v1000.gguf", cfg, seed=5)
    g = Gemma(path, ctx=64)
    o = orc.Model(path, ctx=64, threads=threads, isa="avx512")
    rng = np.random.default_rng(70 + batch)
    H = rng.standard_normal((batch, g.d)).astype(np.float32)
    T = rng.integers(0, g.vocab, batch).astype(np.uint32)
    Hd, Td = torch.tensor(H, device="cuda"), torch.tensor(T.astype(np.int32), device="cuda")
    lp = torch.empty(batch, device="cuda")
    am = torch.empty(batch, dtype=torch.int32, device="cuda")
    g.head_full_dev(Hd.data_ptr(), Td.data_ptr(), batch, lp.data_ptr(), am.data_ptr())
    lp, am = lp.cpu().numpy(), am.cpu().numpy().astype(np.uint32)
    for b in range(batch):
        want = o.full(H[b], int(T[b]))
        assert abs(lp[b] - want[0]) < 2e-5, (b, lp[b], want[0])
        assert am[b] == want[1], b
    g.close()


@pytest.fixture(scope="module")
def f16_head(tmp_path_factory):
    """Q4_0 body with an F16 output matrix of 1000 rows (a partial 64-row tile) and a hidden size of
    352 (two whole 128-column stages and a short third one)."""
    cfg = dict(synth.SMALL, d=352, nh=4, nkv=1, hd=64, ff=512, vocab=1000, layers=2)
    return synth.write_model(tmp_path_factory.mktemp("f16head") / "f16head.gguf", cfg, seed=11, body="q4_0", head="f16")


@pytest.mark.parametrize("n", [1, 33, 300])
def test_parallel_f16_head_full(torch, isa, f16_head, n):
    """The full head of an F16 output matrix as a matrix product (dot16 per row and position) under
    the parallel schedule: one position, a ragged 32-position tile, and two 256-position chunks."""
    from gem_b200 import PARALLEL
    g = Gemma(f16_head, ctx=320)
    g.set_schedule(PARALLEL)
    o = orc.Model(f16_head, ctx=320, threads=REF_THREADS, isa="avx512")
    toks = synth.tokens(n + 1, g.vocab, seed=120 + n)
    lp, am = g.score(toks, FULL)
    lpo, amo, _, _ = o.score(toks, FULL)
    assert np.abs(lp - lpo).max() < 2e-5 and np.array_equal(am, amo), np.abs(lp - lpo).max()
    g.close()


@pytest.mark.parametrize("batch", [5, 13, 40])
def test_head_full_f16_batches(torch, isa, threads, f16_head, batch):
    """Batched full-head calls on an F16 output matrix: streamed per state below 12 states, the
    matrix product from 12 on (a ragged position tile at 13 and 40)."""
    g = Gemma(f16_head, ctx=64)
    o = orc.Model(f16_head, ctx=64, threads=threads, isa="avx512")
    rng = np.random.default_rng(90 + batch)
    H = rng.standard_normal((batch, g.d)).astype(np.float32)
    T = rng.integers(0, g.vocab, batch).astype(np.uint32)
    Hd, Td = torch.tensor(H, device="cuda"), torch.tensor(T.astype(np.int32), device="cuda")
    lp = torch.empty(batch, device="cuda")
    am = torch.empty(batch, dtype=torch.int32, device="cuda")
    g.head_full_dev(Hd.data_ptr(), Td.data_ptr(), batch, lp.data_ptr(), am.data_ptr())
    lp, am = lp.cpu().numpy(), am.cpu().numpy().astype(np.uint32)
    for b in range(batch):
        want = o.full(H[b], int(T[b]))
        assert abs(lp[b] - want[0]) < 2e-5, (b, lp[b], want[0])
        assert am[b] == want[1], b
    g.close()


@pytest.mark.parametrize("which", [-1, 0, 6])
def test_matvec_q4_f16_bit_exact(torch, isa, f16_head, which):
    """The per-token exact GEMV on a Q4_0 body matrix (11 blocks per row: f32 scales) and on an F16
    output matrix (dot16), bit for bit against the oracle's AVX-512 rows."""
    g = Gemma(f16_head, ctx=64)
    name = "token_embd.weight" if which < 0 else f"blk.1.{NAMES[which]}.weight"
    m = _gguf_mat(f16_head, name)
    x = np.random.default_rng(140 + which).standard_normal(m.cols).astype(np.float32)
    xd = torch.tensor(x, device="cuda")
    yd = torch.empty(m.rows, device="cuda")
    g.matvec_dev(1 if which >= 0 else -1, max(which, 0), xd.data_ptr(), yd.data_ptr())
    assert np.array_equal(yd.cpu().numpy().view(np.uint32), m.matvec(x, "avx512", threads=1).view(np.uint32))
    g.close()


def test_sequential_q4_body_f16_head(torch, isa, f16_head):
    """The per-token schedule on a Q4_0 body with an F16 output matrix, against the oracle."""
    from gem_b200 import SEQUENTIAL
    g = Gemma(f16_head, ctx=64)
    g.set_schedule(SEQUENTIAL)
    o = orc.Model(f16_head, ctx=64, threads=REF_THREADS, isa="avx512")
    toks = synth.tokens(30, g.vocab, seed=150)
    lp, am = g.score(toks, FULL)
    lpo, amo, _, _ = o.score(toks, FULL)
    assert np.abs(lp - lpo).max() < 2e-5 and np.array_equal(am, amo), np.abs(lp - lpo).max()
    g.close()


_PARTS_SCRIPT = """
import sys, numpy as np
from gem_b200 import FULL, TWO_LEVEL, Gemma, synth
g = Gemma(sys.argv[1], ctx=600)
g.load_twolevel(sys.argv[2])
toks = synth.tokens(513, g.vocab, seed=160)
lp, am = g.score(toks, TWO_LEVEL)
lpf, amf = g.score(toks, FULL)
np.savez(sys.argv[3], lp=lp, am=am, lpf=lpf, amf=amf)
"""


@pytest.mark.parametrize("parts", [1, 2, 3])
def test_parallel_parts_agree(torch, small, tmp_path, parts):
    """512 positions scored in 1, 2 or 3 parts (uneven: 171 + 171 + 170 positions) give bit-identical
    log-probs and argmax ids to the default 4 parts of 128: the parts change only which stream runs
    which positions. The part count is read once per process, so the other counts run in child
    processes."""
    import os
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    out = tmp_path / f"parts{parts}.npz"
    env = dict(os.environ, GEM_SPLIT=str(parts),
               PYTHONPATH=os.pathsep.join([str(root / "prefix-head_b200"), str(root)]))
    subprocess.run([sys.executable, "-c", _PARTS_SCRIPT, str(small.gguf), str(small.twolevel), str(out)], env=env,
                   check=True, timeout=600)
    got = np.load(out)
    g = Gemma(small.gguf, ctx=600)
    g.load_twolevel(small.twolevel)
    toks = synth.tokens(513, g.vocab, seed=160)
    lp, am = g.score(toks, TWO_LEVEL)
    lpf, amf = g.score(toks, FULL)
    assert np.array_equal(lp.view(np.uint32), got["lp"].view(np.uint32)) and np.array_equal(am, got["am"])
    assert np.array_equal(lpf.view(np.uint32), got["lpf"].view(np.uint32)) and np.array_equal(amf, got["amf"])
    g.close()


@pytest.mark.parametrize("head", [FULL, TWO_LEVEL])
def test_parallel_graph_replay(torch, small, head):
    """A repeated parallel-schedule call replays a CUDA graph of its launches (the second call with the
    same arguments is captured, later ones replay): new token ids in the same buffers give bit-identical
    results to direct calls of a fresh model, across the four streams of a 512-position sequence."""
    def model():
        g = Gemma(small.gguf, ctx=600)
        g.load_twolevel(small.twolevel)
        return g
    a = synth.tokens(513, small.cfg["vocab"], seed=170)
    b = synth.tokens(513, small.cfg["vocab"], seed=171)
    want = {}
    for name, toks in (("a", a), ("b", b)):
        f = model()
        want[name] = f.score(toks, head)  # a fresh model's first call: launched directly
        f.close()
    g = model()
    for name, toks in (("a", a), ("a", a), ("b", b), ("a", a), ("b", b)):  # direct, captured, replays
        lp, am = g.score(toks, head)
        assert np.array_equal(lp.view(np.uint32), want[name][0].view(np.uint32)), name
        assert np.array_equal(am, want[name][1]), name
    g.close()


def test_score_edge_inputs(torch, small):
    """What the reference guards by panicking (an id >= vocab indexes past the embedding, a position
    >= ctx past the KV cache) fails with GEM_E_RANGE before any device work, and the model stays
    usable; an empty sequence scores nothing; the longest sequence ctx allows scores, and its first
    positions equal a short prefix's bit for bit (a position's result depends on no later token)."""
    from gem_b200 import GemError
    ctx = 64
    g = Gemma(small.gguf, ctx=ctx)
    g.load_twolevel(small.twolevel)
    lp, am = g.score(np.array([5], np.uint32), TWO_LEVEL)
    assert lp.shape == (0,) and am.shape == (0,)
    bad = synth.tokens(10, g.vocab, seed=180)
    bad[4] = g.vocab
    with pytest.raises(GemError) as e:
        g.score(bad, FULL)
    assert e.value.code == -7
    with pytest.raises(GemError) as e:
        g.score(synth.tokens(ctx + 2, g.vocab, seed=181), FULL)  # ctx + 1 scored positions
    assert e.value.code == -7
    toks = synth.tokens(ctx + 1, g.vocab, seed=182)  # ctx scored positions: the most ctx holds
    for head in (FULL, TWO_LEVEL):
        lp, am = g.score(toks, head)
        assert lp.shape == (ctx,) and np.all(np.isfinite(lp)) and np.all(lp <= 0)
        lp20, am20 = g.score(toks[:21], head)
        assert np.array_equal(lp[:20].view(np.uint32), lp20.view(np.uint32)) and np.array_equal(am[:20], am20)
    g.close()
