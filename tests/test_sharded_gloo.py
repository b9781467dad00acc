"""Sharded execution over two ranks (gloo, CPU): the group is partitioned by ggemm_shard_group,
each rank computes only its own sub-problems, and the gathered outputs equal the whole group's
outputs bit for bit.

The group is a small image of the BASELINE multi-GPU cases: two operand-reuse components (three
problems sharing each A, as C5's 32 problems share each 4096^2 A), one problem large enough that
the sharder splits it into column blocks (C3's case when problems are fewer than GPUs), and
ragged problems (C2).  Each rank evaluates its pieces with the CPU checker (oracle/, the emulated
DGEMM restated from the reference) on the operands it would hold: the whole A, the B and C
columns of its piece.  Outputs depend per column on that column's own scaling, so a column block
computed alone must reproduce the whole problem's columns exactly.
"""
import os
import socket

import numpy as np
import pytest

import workloads as W

torch = pytest.importorskip("torch")


def mini_group():
    items = []
    for comp in range(2):  # reuse components: A shared by three problems
        for j in range(3):
            items.append(W.Item(96, 40 + 8 * j, 80, 1.0, 1.0, comp, 10 + 3 * comp + j))
    items.append(W.Item(128, 1024, 256, 1.5, 0.0, 2, 20))  # split into column blocks
    for j, (m, n, k) in enumerate([(33, 65, 129), (70, 17, 300), (16, 200, 64)]):
        items.append(W.Item(m, n, k, 0.75, 0.5, 3 + j, 21 + j))
    return W.Workload("mini", items, 2.0, 0, "emu_grouped_reuse", seed=11)


def host_operand(wl, kind, ident, rows, cols):
    rng = np.random.default_rng(W._operand_seed(wl, kind, ident))
    if kind == 2:
        return 2.0 * rng.random((rows, cols)) - 1.0
    return (rng.random((rows, cols)) - 0.5) * np.exp(wl.phi * rng.standard_normal((rows, cols)))


def operands(wl, src):
    it = wl.items[src]
    A = host_operand(wl, 0, it.a, it.m, it.k)
    B = host_operand(wl, 1, it.b, it.k, it.n)
    C = host_operand(wl, 2, src, it.m, it.n)
    return A, B, C


def compute_piece(oracle, wl, src, col0, n):
    """The emulated product of problem src restricted to columns [col0, col0 + n)."""
    it = wl.items[src]
    A, B, C = operands(wl, src)
    N = oracle.choose(it.k, 1e-15)
    Bp = np.ascontiguousarray(B[:, col0:col0 + n].T).reshape(-1)  # column-major, ldb = k
    Cp = np.ascontiguousarray(C[:, col0:col0 + n].T).reshape(-1).copy()
    Af = np.ascontiguousarray(A.T).reshape(-1)
    oracle.emulated(it.m, n, it.k, N, it.alpha, it.beta, Af, it.m, Bp, it.k, Cp, it.m, 1)
    return Cp.reshape(n, it.m).T


def _rank_main(rank, world, port, out_q):
    import torch.distributed as dist

    import g2util

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g2 = g2util.load_pkg()
        oracle = g2util.Oracle()
        wl = mini_group()
        mine = W.shard_pieces(g2, wl, world, rank)
        results = [(p.src, p.col0, p.n, compute_piece(oracle, wl, p.src, p.col0, p.n))
                   for p in mine]
        gathered = [None] * world
        dist.all_gather_object(gathered, results)
        if rank == 0:
            out_q.put(gathered)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_reproduce_the_whole_group(g2, oracle):
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    gathered = q.get(timeout=300)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    wl = mini_group()
    # every column of every problem computed exactly once, and equal to the whole problem
    covered = {i: np.zeros(it.n, dtype=int) for i, it in enumerate(wl.items)}
    ranks_of_component = {}
    split_ranks = set()
    for rank, results in enumerate(gathered):
        assert results, f"rank {rank} got no work"
        for src, col0, n, C in results:
            covered[src][col0:col0 + n] += 1
            whole = compute_piece(oracle, wl, src, 0, wl.items[src].n)
            assert np.array_equal(C.view(np.uint64), whole[:, col0:col0 + n].view(np.uint64)), \
                (src, col0, n)
            if src < 6:
                ranks_of_component.setdefault(wl.items[src].a, set()).add(rank)
            if src == 6:
                split_ranks.add(rank)
    for i, c in covered.items():
        assert np.all(c == 1), f"problem {i} columns covered {c.min()}..{c.max()} times"
    # reuse components stay whole; the large problem spreads over both ranks
    assert all(len(r) == 1 for r in ranks_of_component.values()), ranks_of_component
    assert split_ranks == {0, 1}
