"""gem_head_full_noalloc: the batched full head for callers that cannot allocate device memory when
they score (their memory belongs to another allocator or is planned up front). It must give the same
results as gem_head_full_dev and as the oracle, call after call, through the C ABI, from a single
hidden state up to the largest batch its fixed scratch holds.

This file is named to be collected last, so a stopping run has already run every other test."""
import numpy as np
import pytest

import gem_b200
from gem_b200 import Gemma
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 1 << 20  # the static device array's size (csrc/noalloc.cu)


@pytest.fixture(scope="module")
def torch():
    import torch as t
    if not t.cuda.is_available():
        pytest.skip("no CUDA device")
    return t


def _a16(x):
    return (x + 15) // 16 * 16


def max_fit(d, sms):
    """Largest batch whose quantized states, scales, per-CTA partials and target logits fit the
    scratch: the layout the entry point carves out of its array."""
    parts = 2 * sms
    need = lambda b: _a16(b * d) + _a16(b * (d // 32) * 4) + b * parts * 16 + _a16(b * 4)
    b = 1
    while need(b + 1) <= SCRATCH_BYTES:
        b += 1
    return b


@pytest.mark.parametrize("batch", [1, 11, 16, "max"])
def test_noalloc_head_matches_allocating_head_and_oracle_twice(torch, small, threads, batch):
    g = Gemma(small.gguf, ctx=64)
    if batch == "max":
        batch = max_fit(g.d, torch.cuda.get_device_properties(0).multi_processor_count)
    o = orc.Model(small.gguf, ctx=64, threads=threads, isa="avx512" if orc.detect_isa() == "avx512" else None)
    rng = np.random.default_rng(77 + batch)
    for call in range(2):  # the second call reuses the scratch the first one left behind
        Hh = rng.standard_normal((batch, g.d)).astype(np.float32)
        Th = rng.integers(0, g.vocab, batch).astype(np.uint32)
        H = torch.tensor(Hh, device="cuda")
        T = torch.tensor(Th.astype(np.int32), device="cuda")
        lp_ref = torch.empty(batch, device="cuda")
        am_ref = torch.empty(batch, dtype=torch.int32, device="cuda")
        g.head_full_dev(H.data_ptr(), T.data_ptr(), batch, lp_ref.data_ptr(), am_ref.data_ptr())
        lp = torch.full((batch,), float("nan"), device="cuda")
        am = torch.full((batch,), -1, dtype=torch.int32, device="cuda")
        g.head_full_noalloc(H.data_ptr(), T.data_ptr(), batch, lp.data_ptr(), am.data_ptr())
        g.sync()
        lp, am = lp.cpu().numpy(), am.cpu().numpy().astype(np.uint32)
        np.testing.assert_allclose(lp, lp_ref.cpu().numpy(), rtol=0, atol=2e-5)
        assert np.array_equal(am, am_ref.cpu().numpy().astype(np.uint32)), call
        for b in range(batch):
            want_lp, want_am = o.full(Hh[b], int(Th[b]))
            assert abs(lp[b] - want_lp) < 2e-5, (call, b, lp[b], want_lp)
            if o.isa == "avx512":  # exact numerics reproduce the AVX-512 path's logits bit for bit
                assert am[b] == want_am, (call, b)
    o.close()
    g.close()


def test_noalloc_head_rejects_batches_beyond_its_scratch(torch, small):
    g = Gemma(small.gguf, ctx=64)
    L = gem_b200.lib()
    p = 1 << 20  # never dereferenced: the size check comes first
    rc = L.gem_head_full_noalloc(g.handle, p, p, 100000, p, p)
    assert rc == -1
    assert "scratch" in L.gem_last_error().decode()
    over = max_fit(g.d, torch.cuda.get_device_properties(0).multi_processor_count) + 1
    assert L.gem_head_full_noalloc(g.handle, p, p, over, p, p) == -1  # the first batch that does not fit
    g.close()
