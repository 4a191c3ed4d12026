"""gem_head_full_noalloc: the batched full head for callers that cannot allocate device memory when
they score (their memory belongs to another allocator or is planned up front). It must give the same
results as gem_head_full_dev, call after call, through the C ABI.

This file is named to be collected last, so a stopping run has already run every other test."""
import ctypes as C

import numpy as np
import pytest

import gem_b200
from gem_b200 import Gemma

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    if not t.cuda.is_available():
        pytest.skip("no CUDA device")
    return t


def test_noalloc_head_matches_allocating_head_twice(torch, small):
    g = Gemma(small.gguf, ctx=64)
    rng = np.random.default_rng(77)
    batch = 16
    for call in range(2):
        H = torch.tensor(rng.standard_normal((batch, g.d)).astype(np.float32), device="cuda")
        T = torch.tensor(rng.integers(0, g.vocab, batch).astype(np.int32), device="cuda")
        lp_ref = torch.empty(batch, device="cuda")
        am_ref = torch.empty(batch, dtype=torch.int32, device="cuda")
        g.head_full_dev(H.data_ptr(), T.data_ptr(), batch, lp_ref.data_ptr(), am_ref.data_ptr())
        lp = torch.full((batch,), float("nan"), device="cuda")
        am = torch.full((batch,), -1, dtype=torch.int32, device="cuda")
        g.head_full_noalloc(H.data_ptr(), T.data_ptr(), batch, lp.data_ptr(), am.data_ptr())
        g.sync()
        np.testing.assert_allclose(lp.cpu().numpy(), lp_ref.cpu().numpy(), rtol=0, atol=1e-5)
        assert np.array_equal(am.cpu().numpy(), am_ref.cpu().numpy()), call


def test_noalloc_head_rejects_batches_beyond_its_scratch(torch, small):
    g = Gemma(small.gguf, ctx=64)
    L = gem_b200.lib()
    p = 1 << 20  # never dereferenced: the size check comes first
    rc = L.gem_head_full_noalloc(g.handle, p, p, 100000, p, p)
    assert rc == -1
    assert "scratch" in L.gem_last_error().decode()
