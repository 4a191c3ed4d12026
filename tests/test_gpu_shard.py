"""Vocab-sharded full head through the C ABI: the ranks' merged results equal the unsharded head
(identical argmax ids, log-probs within the log-sum-exp order difference). One rank runs on any GPU
box; two ranks need two GPUs (one process each, NCCL)."""
import os
import socket

import numpy as np
import pytest

from gem_b200 import FULL, TWO_LEVEL, Gemma, nccl_unique_id, synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    if not t.cuda.is_available():
        pytest.skip("no CUDA device")
    return t


def test_single_rank_shard_equals_unsharded(torch, small):
    toks = synth.tokens(70, 8192, seed=31)
    g = Gemma(small.gguf, ctx=128)
    g.load_twolevel(small.twolevel)
    want, want_am = g.score(toks, FULL)
    g.shard(1, 0, nccl_unique_id())
    lp, am = g.score(toks, FULL)
    assert np.abs(lp - want).max() < 2e-5 and np.array_equal(am, want_am)
    lp2, am2 = g.score(toks, TWO_LEVEL)  # the two-level head is unaffected
    g2 = Gemma(small.gguf, ctx=128)
    g2.load_twolevel(small.twolevel)
    w2, wa2 = g2.score(toks, TWO_LEVEL)
    assert np.array_equal(lp2.view(np.uint32), w2.view(np.uint32)) and np.array_equal(am2, wa2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard_worker(rank, world, port, path, twolevel, toks, q):
    import datetime

    import torch
    import torch.distributed as dist
    from gem_b200 import shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        g = Gemma(path, ctx=128, device=rank)
        g.load_twolevel(twolevel)
        rows = shard.init_vocab_shard(g)
        lp, am = g.score(toks, FULL)
        q.put((rank, rows, lp, am))
        g.close()
    finally:
        dist.destroy_process_group()


def test_two_rank_vocab_shard(torch, small):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    toks = synth.tokens(60, 8192, seed=32)
    g = Gemma(small.gguf, ctx=128)
    g.load_twolevel(small.twolevel)
    want, want_am = g.score(toks, FULL)
    g.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_shard_worker, args=(r, 2, port, str(small.gguf), str(small.twolevel), toks, q))
             for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in procs:
        r, rows, lp, am = q.get(timeout=300)
        got[r] = (rows, lp, am)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert got[0][0] == (0, 4096) and got[1][0] == (4096, 4096)
    for r in (0, 1):
        assert np.abs(got[r][1] - want).max() < 2e-5 and np.array_equal(got[r][2], want_am)
