"""Host logic of the multi-GPU paths, on CPU: the vocab-shard row ranges and the data-parallel
sequence split, the communicator-id exchange over a world_size-2 gloo process group, and the merge
of per-shard partial statistics (the algorithm the combine kernel implements) against an unsharded
log-sum-exp / argmax."""
import os
import socket

import numpy as np
import pytest

from gem_b200 import shard


@pytest.mark.parametrize("vocab,n", [(262144, 1), (262144, 2), (262144, 8), (8192, 3), (7, 8)])
def test_row_ranges_partition_the_vocabulary(vocab, n):
    got = [shard.row_range(vocab, n, r) for r in range(n)]
    covered = np.zeros(vocab, int)
    for first, count in got:
        assert count >= 0
        covered[first:first + count] += 1
    assert (covered == 1).all()
    assert all(got[i][0] <= got[i + 1][0] for i in range(n - 1))


@pytest.mark.parametrize("nseq,n", [(256, 1), (256, 8), (10, 4), (3, 8)])
def test_sequence_split(nseq, n):
    got = [shard.seq_range(nseq, n, r) for r in range(n)]
    assert sum(c for _, c in got) == nseq
    assert [f for f, _ in got] == list(np.cumsum([0] + [c for _, c in got[:-1]]))
    assert max(c for _, c in got) - min(c for _, c in got) <= 1


def _merge(parts):
    """The combine kernel's merge: online (max, sum e^(z - max)), best logit (lowest id on ties)."""
    m, s, bv, bt, tl = -np.inf, 0.0, -np.inf, None, None
    for pm, ps, pv, pt, ptl in parts:
        if pm > m:
            s = s * np.exp(m - pm) + ps
            m = pm
        else:
            s = s + ps * np.exp(pm - m)
        if pv > bv or (pv == bv and pt < bt):
            bv, bt = pv, pt
        if not np.isnan(ptl):
            tl = ptl
    return tl - (m + np.log(s)), bt


@pytest.mark.parametrize("n", [1, 2, 3, 8])
def test_shard_merge_equals_unsharded(n):
    rng = np.random.default_rng(n)
    vocab = 1000
    z = rng.standard_normal(vocab) * 3
    z[[17, 900]] = z.max() + 1  # a tie across shards: the lower id wins
    target = 431
    parts = []
    for r in range(n):
        first, count = shard.row_range(vocab, n, r)
        zz = z[first:first + count]
        if count == 0:
            parts.append((-np.inf, 0.0, -np.inf, 2**32 - 1, np.nan))
            continue
        m = zz.max()
        b = int(np.argmax(zz))
        tl = z[target] if first <= target < first + count else np.nan
        parts.append((m, np.exp(zz - m).sum(), zz[b], first + b, tl))
    lp, am = _merge(parts)
    want = z[target] - (z.max() + np.log(np.exp(z - z.max()).sum()))
    assert abs(lp - want) < 1e-9 and am == 17


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exchange_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        uid = bytes(range(128)) if rank == 0 else None
        q.put((rank, shard.exchange_id(uid)))
    finally:
        dist.destroy_process_group()


def test_id_exchange_over_gloo_world_2():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got[0] == got[1] == bytes(range(128))


def test_nccl_unique_id_is_128_bytes():
    import gem_b200
    try:
        a, b = gem_b200.nccl_unique_id(), gem_b200.nccl_unique_id()
    except gem_b200.GemError as e:
        pytest.skip(f"NCCL not loadable here: {e}")
    assert len(a) == len(b) == 128 and a != b
