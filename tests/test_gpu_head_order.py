"""The output matrix held once, in class order (permute_head, crates/gem/src/model.rs:242-249, with
permute_rows, crates/gem/src/q8.rs:65-91).

Loading a two-level class file that covers the vocabulary gathers the output matrix's rows on the device
into class order and releases the token-order rows; the class blocks are views into that one matrix,
and the embedding lookups, the full heads, the vocab shard and the matvec hook find a token's row
through a map. These tests pin that it is one copy and that no result changes: bit-identical to the
oracle (which never permutes) and to a model that loaded only the last class file."""
import numpy as np
import pytest

from gem_b200 import FULL, PARALLEL, SEQUENTIAL, TWO_LEVEL, Gemma, synth
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

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


def test_class_order_keeps_one_copy_of_the_head(torch):
    """Device memory grows by the class table and the maps when the class file loads, not by a second
    178 MB output matrix."""
    mf = synth.ensure("gemma3-270m", classes=2048)
    g = Gemma(mf.gguf, ctx=256)
    head_bytes = g.info["head_bytes"]
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    g.load_twolevel(mf.twolevel)
    torch.cuda.synchronize()
    grown = free_before - torch.cuda.mem_get_info()[0]
    # A (2048 x 640 fp32), b, cls_of, pos_of, order, row_of and the head scratch: ~10 MB
    assert grown < head_bytes // 4, (grown, head_bytes)
    g.close()


def _scores(g, toks):
    out = []
    for sched in (SEQUENTIAL, PARALLEL):
        g.set_schedule(sched)
        for head in (TWO_LEVEL, FULL):
            out.append(g.score(toks, head))
    return out


def test_second_class_file_composes(torch, isa, small, tmp_path):
    """A second class file permutes the already class-ordered rows: results equal a fresh model's that
    loaded only the second file, bit for bit, and the oracle's."""
    g = Gemma(small.gguf, ctx=128)
    g.load_twolevel(small.twolevel)
    tl2 = synth.write_twolevel(tmp_path / "second", g.vocab, 32, g.d, seed=77)
    g.load_twolevel(tl2)
    fresh = Gemma(small.gguf, ctx=128)
    fresh.load_twolevel(tl2)
    toks = synth.tokens(60, g.vocab, seed=21)
    for (lp, am), (lpf, amf) in zip(_scores(g, toks), _scores(fresh, toks)):
        assert np.array_equal(lp.view(np.uint32), lpf.view(np.uint32))
        assert np.array_equal(am, amf)
    o = orc.Model(small.gguf, ctx=128, threads=REF_THREADS, isa="avx512")
    o.load_twolevel(tl2)
    for head in (TWO_LEVEL, FULL):
        lp, am = g.score(toks, head)
        lpo, amo, _, _ = o.score(toks, head)
        assert np.abs(lp - lpo).max() < 2e-5 and np.array_equal(am, amo), head
    o.close()
    fresh.close()
    g.close()


def test_head_matvec_in_token_order_after_permutation(torch, isa, small):
    """gem_matvec_dev on the output matrix returns logits indexed by token whatever the rows' order."""
    g = Gemma(small.gguf, ctx=64)
    x = np.random.default_rng(31).standard_normal(g.d).astype(np.float32)
    xd = torch.tensor(x, device="cuda")
    before = torch.empty(g.vocab, device="cuda")
    g.matvec_dev(-1, 0, xd.data_ptr(), before.data_ptr())
    g.load_twolevel(small.twolevel)
    after = torch.empty(g.vocab, device="cuda")
    g.matvec_dev(-1, 0, xd.data_ptr(), after.data_ptr())
    assert np.array_equal(before.cpu().numpy().view(np.uint32), after.cpu().numpy().view(np.uint32))
    g.close()


def test_partial_class_file_keeps_token_order(torch, isa, small, tmp_path):
    """A class file that covers only part of the vocabulary (the reference gives the other tokens class
    0, position 0: main.rs:66-73) leaves the output matrix in token order and gathers the class blocks
    as a copy; results match the oracle. A covering class file loaded afterwards permutes the matrix and
    releases that copy: bit-identical to a fresh model that loaded only the covering file."""
    import numpy as np
    prefix = tmp_path / "partial"
    rng = np.random.default_rng(41)
    rng.permutation(8000).astype("<u4").tofile(str(prefix) + ".order")
    (rng.standard_normal((64, 256)) * 0.02).astype("<f4").tofile(str(prefix) + ".A")
    np.zeros(64, "<f4").tofile(str(prefix) + ".b")
    g = Gemma(small.gguf, ctx=128)
    g.load_twolevel(prefix)
    o = orc.Model(small.gguf, ctx=128, threads=REF_THREADS, isa="avx512")
    o.load_twolevel(prefix)
    toks = synth.tokens(50, g.vocab, seed=42)
    for head in (TWO_LEVEL, FULL):
        lp, am = g.score(toks, head)
        lpo, amo, _, _ = o.score(toks, head)
        assert np.abs(lp - lpo).max() < 2e-5 and np.array_equal(am, amo), head
    o.close()
    g.load_twolevel(small.twolevel)
    fresh = Gemma(small.gguf, ctx=128)
    fresh.load_twolevel(small.twolevel)
    for (lp, am), (lpf, amf) in zip(_scores(g, toks), _scores(fresh, toks)):
        assert np.array_equal(lp.view(np.uint32), lpf.view(np.uint32)) and np.array_equal(am, amf)
    fresh.close()
    g.close()
