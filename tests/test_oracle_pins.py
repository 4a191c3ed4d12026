"""Pins of the oracle (the CPU restatement of the reference's scoring path) against what anchors it:
the reference's own accuracy tests for its exp/tanh, the llama.cpp block formats via gguf-py, and
restatements of q8.rs's formulas in numpy."""
import numpy as np
import pytest

from oracle import oracle as orc


def test_exp_tanh_match_reference_accuracy_tests():
    # crates/nn/src/fast.rs:206-215: tanh abs err < 2e-6, exp rel err <= 1e-6 * max(1, e^x) on [-10, 10]
    for i in range(-1000, 1001):
        x = np.float32(i / 100.0)
        assert abs(orc.tanh_fast(x) - np.tanh(np.float64(x))) < 2e-6
        e = orc.exp_fast(x)
        assert abs(e - np.exp(np.float64(x))) <= 1e-6 * max(np.exp(np.float64(x)), 1.0)


def test_lse_matches_reference_test_vector():
    # crates/nn/src/fast.rs:216-218: 8193 values ((i*37) % 101)/7 - 5, logsumexp within 1e-4
    v = np.array([((i * 37) % 101) / 7.0 - 5.0 for i in range(8193)], np.float32)
    m = v.max()
    want = m + np.log(np.exp(v.astype(np.float64) - m).sum())
    assert abs(orc.lse(v) - want) < 1e-4


def test_f16_decode_all_bit_patterns():
    # q8.rs:17-26 decodes every f16 exactly, except that exponent 31 (inf and NaN) becomes +-inf
    bits = np.arange(65536, dtype=np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    nan = np.isnan(ref)
    ref[nan] = np.where(bits[nan] & 0x8000, -np.inf, np.inf)
    got = np.array([orc.f16(int(b)) for b in bits], np.float32)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("qtype,kind", [("Q8_0", 8), ("Q4_0", 2)])
def test_block_layout_matches_gguf_py(qtype, kind):
    gguf = pytest.importorskip("gguf")
    from gguf import quants
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((37, 640)) * 0.02).astype(np.float32)
    w[5, :32] = 0.0  # an all-zero block: scale 0
    t = getattr(gguf.GGMLQuantizationType, qtype)
    raw = quants.quantize(w, t)
    want = quants.dequantize(raw, t).reshape(37, 640).astype(np.float32)
    m = orc.Mat(kind, raw, 37, 640)
    got = m.dequant()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_f16_matrix_matches_numpy():
    rng = np.random.default_rng(4)
    w = (rng.standard_normal((9, 96)) * 0.5).astype(np.float16)
    m = orc.Mat(1, w.view(np.uint8).reshape(-1), 9, 96)
    assert np.array_equal(m.dequant(), w.astype(np.float32))


def _round_half_away(x):
    return np.sign(x) * np.floor(np.abs(x) + 0.5)


def test_requantization_formulas():
    # to_q8 (q8.rs:129-145) and to_q4 (q8.rs:148-165) restated in numpy (float32 throughout)
    rng = np.random.default_rng(5)
    w16 = (rng.standard_normal((4, 128)) * 0.03).astype(np.float16)
    m = orc.Mat(1, w16.view(np.uint8).reshape(-1), 4, 128)
    q8 = m.requant(8)
    q, s = q8.planes()
    wf = w16.astype(np.float32).reshape(-1, 32)
    d = (np.abs(wf).max(1) / np.float32(127)).astype(np.float32)
    inv = np.where(d > 0, np.float32(1) / np.where(d > 0, d, 1), 0).astype(np.float32)
    qq = _round_half_away((wf * inv[:, None]).astype(np.float32)).astype(np.int8)
    assert np.array_equal(s, d) and np.array_equal(q.reshape(-1, 32), qq)
    q4 = q8.requant(4)
    q4q, q4s = q4.planes()
    w8 = (qq.astype(np.float32) * d[:, None]).astype(np.float32)
    d4 = (np.abs(w8).max(1) / np.float32(7)).astype(np.float32)
    inv4 = np.where(d4 > 0, np.float32(1) / np.where(d4 > 0, d4, 1), 0).astype(np.float32)
    n = (np.clip(_round_half_away((w8 * inv4[:, None]).astype(np.float32)), -8, 7) + 8).astype(np.uint8)
    packed = (n[:, :16] | (n[:, 16:] << 4)).astype(np.uint8)
    assert np.array_equal(q4s, d4) and np.array_equal(q4q.view(np.uint8).reshape(-1, 16), packed)


@pytest.mark.parametrize("isa", ["avx512", "avx2", "scalar"])
def test_activation_quantize(isa):
    if isa == "avx512" and orc.detect_isa() != "avx512":
        pytest.skip("no AVX-512 on this CPU")
    rng = np.random.default_rng(6)
    x = rng.standard_normal(640).astype(np.float32)
    x[64:96] = 0.0
    q, s = orc.quantize(x, isa)
    xb = x.reshape(-1, 32)
    d = (np.abs(xb).max(1) / np.float32(127)).astype(np.float32)
    inv = np.where(d > 0, np.float32(1) / np.where(d > 0, d, 1), 0).astype(np.float32)
    prod = (xb * inv[:, None]).astype(np.float32)
    want = np.rint(prod) if isa != "scalar" else _round_half_away(prod)  # SIMD: RNE; scalar: round()
    assert np.array_equal(s, d)
    assert np.array_equal(q.reshape(-1, 32), want.astype(np.int8))


@pytest.mark.parametrize("kind,qtype", [(8, "Q8_0"), (2, "Q4_0"), (1, "F16")])
def test_matvec_isa_paths_agree(kind, qtype):
    gguf = pytest.importorskip("gguf")
    from gguf import quants
    rng = np.random.default_rng(7)
    w = (rng.standard_normal((200, 2048)) * 0.02).astype(np.float32)
    raw = w.astype(np.float16).view(np.uint8) if kind == 1 else quants.quantize(w, getattr(gguf.GGMLQuantizationType, qtype))
    m = orc.Mat(kind, raw, 200, 2048)
    x = rng.standard_normal(2048).astype(np.float32)
    ys = {isa: m.matvec(x, isa, threads=3) for isa in ("scalar", "avx2")}
    if orc.detect_isa() == "avx512":
        ys["avx512"] = m.matvec(x, "avx512", threads=3)
    # exact reference: quantized operands in float64
    W = m.dequant().astype(np.float64)
    if kind == 1:
        ref = W @ x.astype(np.float64)
    else:
        q, s = orc.quantize(x, "avx2")
        ref = W @ (q.astype(np.float64) * np.repeat(s, 32))
    for isa, y in ys.items():
        np.testing.assert_allclose(y, ref, rtol=2e-5, atol=2e-6, err_msg=isa)


def test_sampling_generator_is_the_references_xorshift(small):
    """main.rs:123-128: x ^= x << 13; x ^= x >> 7; x ^= x << 17; uniform = (x >> 40) / 2^24. One
    two-level sample draws twice (class, member), so the state advances by two steps."""
    from oracle import oracle as orc
    o = orc.Model(small.gguf, ctx=16, threads=1)
    o.load_twolevel(small.twolevel)
    h = np.random.default_rng(3).standard_normal(o.d).astype(np.float32)
    m = (1 << 64) - 1

    def step(x):
        x ^= (x << 13) & m
        x ^= x >> 7
        x ^= (x << 17) & m
        return x
    seed = 0x0123456789ABCDEF
    _, st = o.sample(h, 1.0, seed)
    assert st == step(step(seed))


def test_greedy_top1_equals_two_level_argmax(small):
    """lean.rs:46-76 with top = 1 and no always-on rows is TwoLevel's argmax (main.rs:101-107 plus the
    screening rule): the same token from both oracle entry points."""
    from oracle import oracle as orc
    o = orc.Model(small.gguf, ctx=16, threads=2)
    o.load_twolevel(small.twolevel)
    rng = np.random.default_rng(4)
    for _ in range(8):
        h = rng.standard_normal(o.d).astype(np.float32)
        assert o.greedy(h, 1)[0] == o.twolevel(h, 0)[1]


@pytest.mark.parametrize("name", ["small", "small-qwen2"])
def test_heads_match_numpy_restatement(name, model_dir):
    """Full::logprob and TwoLevel::logprob (main.rs:20-38, 57-107) restated in float64 numpy on the same
    weights: the head matrix from gguf-py's dequantization times the int8-quantized hidden state
    (Act::quantize, q8.rs:187-246), log-sum-exp over the vocabulary; for the two-level head the class
    files' mapping (per = ceil(V / k), class c holds order[c * per ..]), class logits A h + b on the
    unquantized h, and the target class's block. Agreement within float32 summation noise, and the
    oracle's argmax is a maximum of the restated logits. The qwen2 model's head is its own (untied)
    output matrix."""
    gguf = pytest.importorskip("gguf")
    from gguf import quants
    from gem_b200 import synth
    small = synth.ensure(name, classes=64, directory=model_dir)
    r = gguf.GGUFReader(str(small.gguf))
    names = {t.name: t for t in r.tensors}
    t = names.get("output.weight", names["token_embd.weight"])
    W = np.asarray(quants.dequantize(t.data, t.tensor_type), np.float64).reshape(int(t.shape[1]), int(t.shape[0]))
    V, d = W.shape
    p = str(small.twolevel)
    order = np.fromfile(p + ".order", "<u4").astype(np.int64)
    k = len(np.fromfile(p + ".b", "<f4"))
    A = np.fromfile(p + ".A", "<f4").astype(np.float64).reshape(k, d)
    b = np.fromfile(p + ".b", "<f4").astype(np.float64)
    per = -(-V // k)
    cls_of, pos_of = np.empty(V, np.int64), np.empty(V, np.int64)
    cls_of[order], pos_of[order] = np.arange(V) // per, np.arange(V) % per

    def lse(v):
        m = v.max()
        return m + np.log(np.exp(v - m).sum())

    o = orc.Model(small.gguf, ctx=16, threads=2)
    o.load_twolevel(small.twolevel)
    rng = np.random.default_rng(12)
    for _ in range(6):
        h = rng.standard_normal(d).astype(np.float32)
        q, s = orc.quantize(h, o.isa)
        hq = q.astype(np.float64) * np.repeat(s.astype(np.float64), 32)
        z = W @ hq
        tgt = int(rng.integers(0, V))
        lp, am = o.full(h, tgt)
        assert abs(lp - (z[tgt] - lse(z))) < 2e-4
        assert z.max() - z[am] < 1e-4
        cl = A @ h.astype(np.float64) + b
        c = cls_of[tgt]
        rows = order[c * per:(c + 1) * per]
        inner = W[rows] @ hq
        want = (cl[c] - lse(cl)) + (inner[pos_of[tgt]] - lse(inner))
        lp2, am2 = o.twolevel(h, tgt)
        assert abs(lp2 - want) < 2e-4
        top = int(np.argmax(cl))  # screening with top = 1: the best class, then its best row
        best = W[order[top * per:(top + 1) * per]] @ hq
        assert cls_of[am2] == top or cl.max() - cl[cls_of[am2]] < 1e-4
        if cls_of[am2] == top:
            assert best.max() - best[pos_of[am2]] < 1e-4
