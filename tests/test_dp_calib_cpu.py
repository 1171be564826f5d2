"""Data-parallel calibration's early stop, on CPU ranks over gloo.

CausalProfiler(dp_group=...) splits the calibration batches over the ranks,
and every rank must take the Spearman early-stop decision of
csaq/core.py:212-230 on the same numbers: rank 0 draws the sample indices
and broadcasts them, each rank gathers its own salience at those indices
(layer by layer, without concatenating every layer's salience), and the
sample is summed over the ranks before ranking. Two gloo processes hold
complementary halves of a set of layer salience accumulators; their
all-reduced sample must equal the single-process sample of the summed
salience, element for element, and give the same rho. No GPU is used.
"""

import os
import socket
from types import SimpleNamespace

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


SHAPES = {"a": (40, 24), "b": (17, 31), "c": (64, 8)}


def _salience(step: int, part: int):
    """Per-layer accumulators of rank `part` after `step` evaluations (integer
    valued, so sums over ranks are exact in fp32)."""
    g = torch.Generator().manual_seed(100 * step + part)
    return {n: torch.randint(0, 1000, s, generator=g).float() for n, s in SHAPES.items()}


def _profiler(sal, group, sample: int):
    from csaq.core import CausalProfiler
    return SimpleNamespace(salience=sal, _modules={n: None for n in SHAPES}, dp_group=group,
                           _SPEARMAN_SAMPLE=sample, _RANDPERM_MAX=CausalProfiler._RANDPERM_MAX,
                           _spearman_indices=None)


def _sample_once(sal, group, world, sample, idx=None):
    from csaq.core import CausalProfiler
    p = _profiler(sal, group, sample)
    if idx is None:
        torch.manual_seed(5)
        idx = CausalProfiler._spearman_indices(p, torch.device("cpu"), dist if world > 1 else None, world)
    s = CausalProfiler._salience_sample(p, idx, torch.device("cpu"))
    if world > 1:
        dist.all_reduce(s, group=group)
    return idx, s


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from csaq.core import spearman_rho
        out = []
        prev = None
        idx = None
        for step in range(2):
            idx, s = _sample_once(_salience(step, rank), dist.group.WORLD, world, 500, idx)
            r = s.argsort().argsort().float()
            # plain lists: a tensor on the queue is a shared-memory handle that dies with this process
            out.append((idx.tolist(), s.tolist(), None if prev is None else spearman_rho(r, prev)))
            prev = r
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_dp_spearman_sample_equals_single_process():
    from csaq.core import spearman_rho
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, out = q.get(timeout=300)
        res[rank] = [(torch.tensor(i), torch.tensor(v), rho) for i, v, rho in out]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # every rank drew nothing itself but received rank 0's indices, and summed the same sample
    for step in range(2):
        assert torch.equal(res[0][step][0], res[1][step][0])
        assert torch.equal(res[0][step][1], res[1][step][1])
    # single process over the summed salience: the same indices give the same sample and rho
    prev, idx = None, res[0][0][0]
    for step in range(2):
        tot = {n: _salience(step, 0)[n] + _salience(step, 1)[n] for n in SHAPES}
        _, s = _sample_once(tot, None, 1, 500, idx)
        assert torch.equal(s, res[0][step][1])
        r = s.argsort().argsort().float()
        if prev is not None:
            assert spearman_rho(r, prev) == res[0][step][2]
        prev = r
    # the sample without the concatenation is the reference's all_s[idx]
    tot = {n: _salience(0, 0)[n] + _salience(0, 1)[n] for n in SHAPES}
    all_s = torch.cat([tot[n].flatten() for n in SHAPES])
    assert torch.equal(all_s[idx], _sample_once(tot, None, 1, 500, idx)[1])


def test_spearman_indices_follow_the_reference_draw():
    """Below the size cap the sample is torch.randperm(N)[:size] on the host
    generator, as csaq/core.py:214-216 draws it."""
    from csaq.core import CausalProfiler
    sal = _salience(0, 0)
    p = _profiler(sal, None, 300)
    N = sum(t.numel() for t in sal.values())
    torch.manual_seed(9)
    ref = torch.randperm(N)[:300]
    torch.manual_seed(9)
    got = CausalProfiler._spearman_indices(p, torch.device("cpu"), None, 1)
    assert torch.equal(ref, got)
    # above the cap: distinct indices, all in range
    p._RANDPERM_MAX = 10
    got = CausalProfiler._spearman_indices(p, torch.device("cpu"), None, 1)
    assert got.numel() == 300 and got.unique().numel() == 300 and int(got.min()) >= 0 and int(got.max()) < N
