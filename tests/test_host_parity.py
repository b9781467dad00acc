"""Host logic against the reference's own host code (CPU only).

Planner: route, moduli count and tile class per problem equal the reference planner
(src/planner.cpp:286-330, built in oracle/_ref) for the same device model, including its
route test table (tests/test_planner.cpp:127-176).  Operand reuse: unique-operand numbering,
per-operand N, promotion (src/operand_reuse.cpp:47-141).  Sharder: structural properties.
"""
import ctypes

import numpy as np
import pytest

KMAX = 131040


def _problems(g2, specs):
    return g2.make_problems([dict(m=m, n=n, k=k, A=A, lda=lda, B=B, ldb=ldb, C=C, ldc=ldc,
                                  alpha=alpha, beta=beta)
                             for (m, n, k, A, lda, B, ldb, C, ldc, alpha, beta) in specs])


def _spec(m, n, k, alpha=1.0, beta=0.0, A=0x1000, B=0x2000, C=0x3000):
    return (m, n, k, A, max(1, m), B, max(1, k), C, max(1, m), alpha, beta)


DM = dict(num_sms=148, fp64=36e12, int8=2.5e15, bw=6.0e12, tiny=32768.0)


def plan_both(g2, ref, specs, cfg, path, dm=DM, rho=16.0):
    P = _problems(g2, specs)
    num = len(specs)
    r1, n1, t1 = (ctypes.c_int * max(1, num))(), (ctypes.c_int * max(1, num))(), (ctypes.c_int * max(1, num))()
    rc1 = g2.lib.ggemm_stage_plan(P, num, ctypes.byref(cfg), path, dm["num_sms"], dm["fp64"],
                                  dm["int8"], dm["bw"], dm["tiny"], rho, r1, n1, t1)
    entry = ctypes.c_byte * ref.L.ozr_sizeof_plan_entry()
    out = (entry * max(1, num))()
    rc2 = ref.L.ozr_plan(ctypes.cast(P, ctypes.c_void_p), num, ctypes.addressof(cfg), path,
                         dm["num_sms"], dm["fp64"], dm["int8"], dm["bw"], dm["tiny"],
                         ctypes.addressof(out))
    mine = [(r1[i], n1[i]) for i in range(num)]
    theirs = []
    for i in range(num):
        raw = bytes(out[i])
        route, nm, tile = np.frombuffer(raw[:12], dtype=np.int32)
        theirs.append((int(route), int(nm)))
    return rc1, rc2, mine, theirs


EMU, UNPROFITABLE = 0, 5


def same_plan(mine, theirs):
    """Rule routes (empty, k = 0, alpha = 0, k too large, small k, precision, tiny) and moduli
    counts equal the reference's; where the reference's H200 throughput model decides (emulate or
    UNPROFITABLE), this library's calibrated B200 model may decide either way."""
    for (r, n), (R, N) in zip(mine, theirs):
        assert n == N, (r, n, R, N)
        if R in (EMU, UNPROFITABLE):
            assert r in (EMU, UNPROFITABLE), (r, R)
        else:
            assert r == R, (r, R)


ROUTE_CASES = [
    # (m, n, k, alpha, beta), num_moduli, allow_fallback, path
    ((256, 256, KMAX + 1), 0, 1, 4), ((256, 256, KMAX + 1), 0, 1, 3), ((256, 256, 200000), 8, 1, 4),
    ((256, 256, KMAX + 1), 0, 0, 4), ((256, 256, KMAX + 1), 0, 0, 2), ((256, 256, KMAX + 1), 8, 0, 3),
    ((256, 256, KMAX), 0, 0, 4), ((512, 512, 1), 0, 1, 4), ((512, 512, 16), 0, 1, 4),
    ((512, 512, 17), 0, 1, 4), ((512, 512, 8), 0, 0, 4), ((512, 512, 8), 0, 1, 3),
    ((512, 512, 512, 0.0, 1.0), 0, 1, 4), ((512, 512, 512, 0.0, 0.5), 0, 0, 4),
    ((512, 512, 512, 0.0, 0.0), 4, 0, 3), ((512, 512, 8, 0.0, 1.0), 0, 1, 4),
    ((0, 512, 512), 0, 0, 4), ((512, 0, 512), 0, 1, 3), ((512, 512, 0), 0, 1, 4),
    ((8192, 8192, 8192), 0, 1, 4), ((16, 16, 16), 0, 1, 4), ((20, 20, 20), 0, 1, 4),
]


@pytest.mark.parametrize("case", ROUTE_CASES)
def test_planner_routes_match_reference(g2, ref, case):
    shape, nm, fb, path = case
    spec = _spec(*shape)
    cfg = g2.Config(nm, 1e-15, fb, 0)
    rc1, rc2, mine, theirs = plan_both(g2, ref, [spec], cfg, path)
    assert rc1 == rc2
    if rc1 == 0:
        same_plan(mine, theirs)


@pytest.mark.parametrize("path", [2, 3, 4])
@pytest.mark.parametrize("seed", [1, 2, 3])
def test_planner_random_groups_match_reference(g2, ref, path, seed):
    rng = np.random.default_rng(seed)
    specs = []
    for i in range(200):
        m, n = (int(x) for x in np.exp(rng.uniform(np.log(1), np.log(3000), 2)))
        k = int(np.exp(rng.uniform(0, np.log(140000))))
        if rng.random() < 0.05:
            k = 0
        alpha = 0.0 if rng.random() < 0.05 else float(rng.uniform(0.5, 2))
        beta = 0.0 if rng.random() < 0.5 else 0.5
        specs.append(_spec(m, n, k, alpha, beta))
    for cfg in (g2.Config(0, 1e-15, 1, 0), g2.Config(12, 1e-15, 1, 0), g2.Config(0, 1e-12, 1, 0),
                g2.Config(0, 1e-15, 0, 0)):
        for dm in (DM, dict(num_sms=132, fp64=53.6e12, int8=0.99e15, bw=2.68e12, tiny=32768.0)):
            rc1, rc2, mine, theirs = plan_both(g2, ref, specs, cfg, path, dm)
            assert rc1 == rc2
            if rc1 == 0:
                if path == 4:
                    same_plan(mine, theirs)
                else:  # no cost model involved: every route by rule
                    assert mine == theirs


def _reuse_both(g2, ref, specs, nmod, policy):
    P = _problems(g2, specs)
    num = len(specs)
    nm = (ctypes.c_int * num)(*nmod)
    o1 = (ctypes.c_int * (3 + 7 * num))()
    o2 = (ctypes.c_int * (3 + 7 * num))()
    assert g2.lib.ggemm_stage_reuse(P, num, nm, policy, o1) == 0
    assert ref.L.ozr_reuse(ctypes.cast(P, ctypes.c_void_p), num, ctypes.addressof(nm), policy,
                           ctypes.addressof(o2)) == 0
    return list(o1), list(o2)


@pytest.mark.parametrize("policy", [0, 1])
@pytest.mark.parametrize("seed", [11, 12, 13])
def test_reuse_matches_reference(g2, ref, policy, seed):
    rng = np.random.default_rng(seed)
    specs, nmod = [], []
    As = [0x10000 * (i + 1) for i in range(6)]
    Bs = [0x100000000 * (i + 1) for i in range(6)]
    for g in range(120):
        a, b = int(rng.integers(0, 6)), int(rng.integers(0, 6))
        k = [64, 128, 256][a % 3]
        specs.append(_spec(100 + a, 50 + b, k, 1.0, 0.0, A=As[a], B=Bs[b]))
        nmod.append(int(rng.choice([0, 14, 15, 16])))
    o1, o2 = _reuse_both(g2, ref, specs, nmod, policy)
    assert o1 == o2


@pytest.mark.parametrize("policy", [0, 1])
@pytest.mark.parametrize("seed", [21, 22, 23, 24])
def test_reuse_matches_reference_sparse_chains(g2, ref, policy, seed):
    """Many operands, sparse sharing (long promotion chains A - B - A ...), one pointer under
    several (ld, rows, k) keys, and problems that are not emulated (nmod 0)."""
    rng = np.random.default_rng(seed)
    specs, nmod = [], []
    for g in range(400):
        a, b = int(rng.integers(0, 60)), int(rng.integers(0, 60))
        k = [64, 96][int(rng.integers(0, 2))]
        m = 40 + (a % 5)
        lda = m + int(rng.integers(0, 2))
        spec = list(_spec(m, 30 + b % 7, k, 1.0, 0.0, A=0x10000 * (a + 1), B=0x1000000 * (b + 1)))
        spec[4] = lda
        specs.append(tuple(spec))
        nmod.append(int(rng.choice([0, 8, 14, 15, 16, 20])))
    o1, o2 = _reuse_both(g2, ref, specs, nmod, policy)
    assert o1 == o2


def test_reuse_c5_pattern(g2, ref):
    """Config 5 shape: 16 shared A, 32 distinct B each -> 16 unique A, 512 unique B."""
    specs = [_spec(4096, 1024, 4096, 1.0, 1.0, A=0x1000 * (1 + g // 32), B=0x100000 * (g + 1))
             for g in range(512)]
    o1, o2 = _reuse_both(g2, ref, specs, [15] * 512, 0)
    assert o1 == o2
    assert o1[0] == 16 and o1[1] == 512


def _shard(g2, specs, S):
    P = _problems(g2, specs)
    return g2.shard_group(P, len(specs), S)


@pytest.mark.parametrize("S", [1, 2, 4, 8])
def test_shard_partition_properties(g2, S):
    rng = np.random.default_rng(S)
    specs = [_spec(int(rng.integers(128, 2049)), int(rng.integers(128, 2049)),
                   int(rng.integers(128, 2049)), 1.0, 0.5, A=0x1000 * (g + 1),
                   B=0x10000000 * (g + 1), C=0x1000000000 * (g + 1)) for g in range(64)]
    subs, shard, src = _shard(g2, specs, S)
    cover = {}
    for i, g in enumerate(src):
        p = subs[i]
        j0 = (p.C - specs[g][7]) // 8 // specs[g][8]
        cover.setdefault(g, []).append((j0, j0 + p.n, shard[i]))
        assert p.m == specs[g][0] and p.k == specs[g][2]
    for g, blocks in cover.items():
        blocks.sort()
        assert blocks[0][0] == 0 and blocks[-1][1] == specs[g][1]
        for a, b in zip(blocks, blocks[1:]):
            assert a[1] == b[0]
    assert set(cover) == set(range(64))
    cost = [0.0] * S
    for i, g in enumerate(src):
        cost[shard[i]] += subs[i].m * subs[i].n * subs[i].k
    assert max(cost) <= 1.25 * (sum(cost) / S)


def test_shard_keeps_shared_operands_together(g2):
    """Config 5: 16 A components x 32 problems over 8 shards -> 2 components per shard."""
    specs = [_spec(4096, 1024, 4096, 1.0, 1.0, A=0x1000 * (1 + g // 32), B=0x100000 * (g + 1),
                   C=0x100000000 * (g + 1)) for g in range(512)]
    subs, shard, src = _shard(g2, specs, 8)
    comp_shard = {}
    for i, g in enumerate(src):
        comp_shard.setdefault(g // 32, set()).add(shard[i])
    assert all(len(s) == 1 for s in comp_shard.values())
    per = [sum(1 for s in comp_shard.values() if x in s) for x in range(8)]
    assert per == [2] * 8


def test_shard_splits_large_problems(g2):
    """Config 3: 8 x 8192^3 over 8 shards -> one problem per shard; 1 problem over 4 -> columns."""
    specs = [_spec(8192, 8192, 8192, A=0x1000 * (g + 1), B=0x100000 * (g + 1),
                   C=0x100000000 * (g + 1)) for g in range(8)]
    subs, shard, src = _shard(g2, specs, 8)
    assert sorted(shard) == list(range(8)) and len(shard) == 8
    subs, shard, src = _shard(g2, specs[:1], 4)
    assert sorted(set(shard)) == [0, 1, 2, 3]
    assert sum(subs[i].n for i in range(len(shard))) == 8192
