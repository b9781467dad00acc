"""Sharded run on two GPUs equals the single-GPU run, bit for bit.

Two processes (one per GPU) each take the sub-problems ggemm_shard_group gives their shard, hold
the operands those touch (tests/workloads.py regenerates them from per-operand seeds) and run
ggemm_grouped_dgemm on their own device; the parent then runs the whole group on one GPU and
compares every output column.  The group mixes operand-reuse components (EMU_GROUPED_REUSE, as
in C5) with one problem large enough to be split into column blocks across the GPUs (C3's case
when problems are fewer than GPUs).  Skipped on a machine with fewer than two GPUs.  No
collective is involved: outputs are disjoint.
"""
import numpy as np
import pytest

import workloads as W

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def group():
    items = []
    for comp in range(4):
        for j in range(6):
            items.append(W.Item(512, 256 + 64 * j, 384, 1.0, 1.0, comp, 100 + 10 * comp + j))
    items.append(W.Item(2048, 8192, 2048, 1.5, 0.5, 9, 200))
    return W.Workload("multi", items, 1.0, 0, "emu_grouped_reuse", seed=21)


def run_pieces(g2, wl, pieces, device):
    grp = W.DeviceGroup(g2, wl, pieces, device)
    cfg = g2.config(0, 1e-15, 1, 0)
    with g2.Handle(grp.num, grp.budget[0] + 1, grp.budget[1] + 1, grp.budget[2] + 1,
                   stream=torch.cuda.current_stream(device).cuda_stream) as h:
        rc, _ = h.grouped_dgemm(g2.PATH_EMU_GROUPED_REUSE, cfg, grp.problems, grp.num)
        torch.cuda.synchronize(device)
        assert rc == 0 and h.device_status() == 0
    out = []
    for p in pieces:
        it = wl.items[p.src]
        C = grp.output(p.src).view(it.n, it.m)[p.col0:p.col0 + p.n].cpu().numpy()
        out.append((p.src, p.col0, p.n, C))
    return out


def _worker(rank, world, q):
    import g2util

    torch.cuda.set_device(rank)
    g2 = g2util.load_pkg()
    wl = group()
    pieces = W.shard_pieces(g2, wl, world, rank)
    q.put((rank, run_pieces(g2, wl, pieces, torch.device("cuda", rank))))


def test_two_gpus_reproduce_single_gpu(g2, cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    wl = group()
    whole = {src: C for src, _, _, C in run_pieces(g2, wl, W.shard_pieces(g2, wl, 1, 0),
                                                   torch.device("cuda", 0))}
    covered = {i: np.zeros(it.n, dtype=int) for i, it in enumerate(wl.items)}
    split = set()
    for rank in range(world):
        assert results[rank], f"GPU {rank} got no work"
        for src, col0, n, C in results[rank]:
            covered[src][col0:col0 + n] += 1
            assert np.array_equal(C.view(np.uint64), whole[src][col0:col0 + n].view(np.uint64)), \
                (rank, src, col0)
            if src == len(wl.items) - 1:
                split.add(rank)
    assert all(np.all(c == 1) for c in covered.values())
    assert split == {0, 1}  # the large problem spreads over both GPUs
