"""Seeded synthetic groups of the five BASELINE configurations (C1 .. C5), shared by bench.py and
the at-size parity tests.

Every configuration is a list of problems whose A and B operands carry ids: problems that share
an operand (C5: 32 problems per A matrix) name the same id, and the bytes of an operand depend only
on (configuration seed, operand id).  A shard of the group (ggemm_shard_group) therefore
regenerates exactly the bytes the whole group holds, on any GPU, and the sharded outputs can be
compared with the single-GPU outputs bit for bit.

Entry distributions follow the reference's convention a = (U(0,1) - 0.5) exp(phi N(0,1))
(bench/workloads.h:26-27); C1 uses U[-1, 1) as its configuration states.  These are synthetic
inputs of the configurations' shapes and distributions (no dataset is involved); the generator
is torch's Philox on the device, seeded per operand.

  C1  4 x 256^3, A, B, C ~ U[-1, 1), alpha 1, beta 0, N = 14, allow_fallback 1
  C2  64 ragged problems, m, n, k uniform over {128, 192, ..., 2048}, phi 2, alpha ~ U(0.5, 2),
      beta 0.5, C ~ U[-1, 1), adaptive N (target 1e-15)
  C3  8 x 8192^3, phi 0.5, alpha 1, beta 0, N = 16
  C4  1024 skewed problems, m, n log-uniform [16, 512], k log-uniform [16, 4096], phi 4, 0.1 % of
      A entries NaN / +Inf at seeded positions, 5 % of problems alpha = 0 (the others alpha ~
      U(0.5, 2)), beta 0.5, C ~ U[-1, 1), adaptive N, handle min_k 16
  C5  16 A matrices 4096 x 4096, each shared by 32 problems with their own B (4096 x 1024), phi 1,
      alpha 1, beta 1, C ~ U[-1, 1), adaptive N, operand reuse (EMU_GROUPED_REUSE)
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

C2_SIZES = list(range(128, 2049, 64))
C2_SEED = 20261201  # shape seed of the C2 group (the bench workload of earlier measurements)


@dataclass
class Item:
    m: int
    n: int
    k: int
    alpha: float
    beta: float
    a: int  # A operand id (problems sharing an A matrix share the id)
    b: int  # B operand id


@dataclass
class Workload:
    name: str
    items: list
    phi: float | None  # None: U[-1, 1) entries (C1)
    num_moduli: int
    path_name: str
    min_k: int = 32
    nonfinite_frac: float = 0.0  # fraction of A entries set to NaN / +Inf
    seed: int = 0
    scaling: str = "strong"  # how the group spreads over N GPUs (bench.py)
    describe: str = ""
    allow_fallback: int = 1
    target_rel_err: float = 1e-15
    a_shape: dict = field(default_factory=dict)  # id -> (rows, k)
    b_shape: dict = field(default_factory=dict)  # id -> (k, cols)

    def __post_init__(self):
        for it in self.items:
            self.a_shape.setdefault(it.a, (it.m, it.k))
            self.b_shape.setdefault(it.b, (it.k, it.n))

    @property
    def flops(self) -> float:
        return sum(2.0 * it.m * it.n * it.k for it in self.items)

    def elems(self):
        """(A, B, C) elements the public call's budgets count (sum over problems)."""
        return (sum(it.m * it.k for it in self.items), sum(it.k * it.n for it in self.items),
                sum(it.m * it.n for it in self.items))


# --------------------------------------------------------------------------------- configs
def c1() -> Workload:
    items = [Item(256, 256, 256, 1.0, 0.0, g, g) for g in range(4)]
    return Workload("c1", items, None, 14, "emu_grouped", seed=0, scaling="weak",
                    describe="C1: G=4 x 256^3, A,B,C ~ U[-1,1) seed 0, alpha=1 beta=0, N=14, "
                             "allow_fallback=1")


def c2_items(num: int, seed: int = C2_SEED):
    rng = np.random.default_rng(seed)
    m = rng.choice(C2_SIZES, num)
    n = rng.choice(C2_SIZES, num)
    k = rng.choice(C2_SIZES, num)
    alpha = rng.uniform(0.5, 2.0, num)
    return [Item(int(m[i]), int(n[i]), int(k[i]), float(alpha[i]), 0.5, i, i)
            for i in range(num)]


def c2(num: int = 64, seed: int = C2_SEED) -> Workload:
    return Workload("c2", c2_items(num, seed), 2.0, 0, "emu_grouped", seed=seed, scaling="weak",
                    describe=f"C2: G={num} ragged m,n,k uniform in {{128..2048 step 64}}, phi=2, "
                             "alpha~U(0.5,2), beta=0.5, C~U[-1,1), adaptive N (target 1e-15)")


def c3(num: int = 8) -> Workload:
    items = [Item(8192, 8192, 8192, 1.0, 0.0, g, g) for g in range(num)]
    return Workload("c3", items, 0.5, 16, "emu_grouped", seed=3, scaling="strong",
                    describe=f"C3: G={num} x 8192^3, phi=0.5, alpha=1 beta=0, N=16")


def _log_uniform(rng, lo, hi, size):
    x = np.exp(rng.uniform(math.log(lo), math.log(hi), size))
    return np.clip(np.rint(x).astype(np.int64), lo, hi)


def c4(num: int = 1024, seed: int = 4) -> Workload:
    rng = np.random.default_rng(seed)
    m = _log_uniform(rng, 16, 512, num)
    n = _log_uniform(rng, 16, 512, num)
    k = _log_uniform(rng, 16, 4096, num)
    alpha = rng.uniform(0.5, 2.0, num)
    zero = rng.choice(num, int(round(0.05 * num)), replace=False)
    alpha[zero] = 0.0
    items = [Item(int(m[i]), int(n[i]), int(k[i]), float(alpha[i]), 0.5, i, i)
             for i in range(num)]
    return Workload("c4", items, 4.0, 0, "auto", min_k=16, nonfinite_frac=1e-3, seed=seed,
                    scaling="strong",
                    describe=f"C4: G={num} skewed, m,n log-uniform [16,512], k log-uniform "
                             "[16,4096], phi=4, 0.1% of A entries NaN/+Inf, 5% alpha=0, "
                             "beta=0.5, adaptive N, min_k=16")


def c5(components: int = 16, per: int = 32) -> Workload:
    items = []
    for c in range(components):
        for j in range(per):
            p = c * per + j
            items.append(Item(4096, 1024, 4096, 1.0, 1.0, c, p))
    return Workload("c5", items, 1.0, 0, "emu_grouped_reuse", seed=5, scaling="strong",
                    describe=f"C5: G={components * per}, {components} shared A 4096x4096 x {per} "
                             "problems each with distinct B 4096x1024, phi=1, alpha=1 beta=1, "
                             "C~U[-1,1), adaptive N, operand reuse")


CONFIGS = {"c1": c1, "c2": c2, "c3": c3, "c4": c4, "c5": c5}


# -------------------------------------------------------------------------------- sharding
_A_BASE, _B_BASE, _C_BASE, _SPAN = 1 << 40, 1 << 50, 1 << 56, 1 << 36


def logical_problems(g2, wl: Workload):
    """The group with stand-in pointers (one per operand id, 64 GiB apart) for the sharder,
    which looks at pointers only to find shared operands and to offset column blocks."""
    return g2.make_problems([dict(m=it.m, n=it.n, k=it.k, A=_A_BASE + it.a * _SPAN, lda=it.m,
                                  B=_B_BASE + it.b * _SPAN, ldb=it.k,
                                  C=_C_BASE + i * _SPAN, ldc=it.m, alpha=it.alpha,
                                  beta=it.beta)
                             for i, it in enumerate(wl.items)])


@dataclass
class Piece:
    src: int   # problem of the group
    col0: int  # first column of the piece
    n: int     # its columns


def shard_pieces(g2, wl: Workload, world: int, rank: int):
    """The pieces of the group that ggemm_shard_group gives shard `rank` of `world`."""
    if world == 1:
        return [Piece(i, 0, it.n) for i, it in enumerate(wl.items)]
    logical = logical_problems(g2, wl)
    subs, shard, src = g2.shard_group(logical, len(wl.items), world)
    out = []
    for i in range(len(shard)):
        if shard[i] != rank:
            continue
        s = src[i]
        col0 = (subs[i].C - logical[s].C) // (8 * wl.items[s].m)
        out.append(Piece(s, int(col0), int(subs[i].n)))
    return out


# ------------------------------------------------------------------------------ device data
def _operand_seed(wl: Workload, kind: int, ident: int) -> int:
    return (wl.seed * 1000003 + kind * 7919 + ident * 104729 + 12345) & 0x7FFFFFFFFFFF


def fill(t, wl: Workload, kind: int, ident: int, nonfinite: float = 0.0):
    """Entries of operand `ident` (kind 0 = A, 1 = B, 2 = C) in place, from its own seed."""
    import torch

    g = torch.Generator(device=t.device)
    g.manual_seed(_operand_seed(wl, kind, ident))
    u = torch.rand(t.shape, generator=g, device=t.device, dtype=torch.float64)
    if kind == 2 or wl.phi is None:
        t.copy_(2.0 * u - 1.0)  # U[-1, 1)
    elif wl.phi == 0.0:
        t.copy_(u - 0.5)
    else:
        z = torch.randn(t.shape, generator=g, device=t.device, dtype=torch.float64)
        t.copy_((u - 0.5) * torch.exp(wl.phi * z))
    if nonfinite > 0.0:
        hit = torch.rand(t.shape, generator=g, device=t.device, dtype=torch.float64) < nonfinite
        kind_nan = torch.rand(t.shape, generator=g, device=t.device, dtype=torch.float64) < 0.5
        t.masked_fill_(hit & kind_nan, float("nan"))
        t.masked_fill_(hit & ~kind_nan, float("inf"))


class DeviceGroup:
    """Device buffers of the pieces one rank runs: every A and B operand they touch (whole, with
    tight leading dimensions), every C they touch (whole), and the problem descriptors.
    c0 keeps a device copy of the initial C (for resets and parity checks)."""

    def __init__(self, g2, wl: Workload, pieces, device, keep_c0: bool = False):
        import torch

        self.g2, self.wl, self.pieces, self.device = g2, wl, pieces, device
        a_ids = sorted({wl.items[p.src].a for p in pieces})
        b_ids = sorted({wl.items[p.src].b for p in pieces})
        c_ids = sorted({p.src for p in pieces})
        self.a_off, self.b_off, self.c_off = {}, {}, {}
        na = nb = nc = 0
        for a in a_ids:
            self.a_off[a] = na
            r, k = wl.a_shape[a]
            na += r * k
        for b in b_ids:
            self.b_off[b] = nb
            k, c = wl.b_shape[b]
            nb += k * c
        for s in c_ids:
            self.c_off[s] = nc
            nc += wl.items[s].m * wl.items[s].n
        self.na, self.nb, self.nc = na, nb, nc
        f64 = torch.float64
        self.A = torch.empty(max(na, 1), dtype=f64, device=device)
        self.B = torch.empty(max(nb, 1), dtype=f64, device=device)
        self.C = torch.empty(max(nc, 1), dtype=f64, device=device)
        for a in a_ids:
            r, k = wl.a_shape[a]
            fill(self.A[self.a_off[a]:self.a_off[a] + r * k], wl, 0, a, wl.nonfinite_frac)
        for b in b_ids:
            k, c = wl.b_shape[b]
            fill(self.B[self.b_off[b]:self.b_off[b] + k * c], wl, 1, b)
        for s in c_ids:
            mn = wl.items[s].m * wl.items[s].n
            fill(self.C[self.c_off[s]:self.c_off[s] + mn], wl, 2, s)
        self.c0 = self.C.clone() if keep_c0 else None
        self.num = len(pieces)
        self.problems = self.problems_on(self.A, self.B, self.C)
        # budgets of the public call (sums over problems, as ggemm_create's element counts)
        self.budget = (sum(wl.items[p.src].m * wl.items[p.src].k for p in pieces),
                       sum(wl.items[p.src].k * p.n for p in pieces),
                       sum(wl.items[p.src].m * p.n for p in pieces))
        self.flops = sum(2.0 * wl.items[p.src].m * p.n * wl.items[p.src].k for p in pieces)

    def entries_on(self, A, B, C):
        out = []
        for p in self.pieces:
            it = self.wl.items[p.src]
            out.append(dict(m=it.m, n=p.n, k=it.k,
                            A=A.data_ptr() + 8 * self.a_off[it.a], lda=it.m,
                            B=B.data_ptr() + 8 * (self.b_off[it.b] + p.col0 * it.k), ldb=it.k,
                            C=C.data_ptr() + 8 * (self.c_off[p.src] + p.col0 * it.m), ldc=it.m,
                            alpha=it.alpha, beta=it.beta))
        return out

    def problems_on(self, A, B, C):
        """The same problems with their operands in other device buffers of the same sizes."""
        return self.g2.make_problems(self.entries_on(A, B, C))

    def reset(self):
        self.C.copy_(self.c0)

    def shapes(self):
        """(m, n, k, alpha, beta) per piece."""
        return [(self.wl.items[p.src].m, p.n, self.wl.items[p.src].k, self.wl.items[p.src].alpha,
                 self.wl.items[p.src].beta) for p in self.pieces]

    def unique_shapes(self):
        """(rows, k) of each unique A operand and (k, cols) of each unique B operand held."""
        return ([self.wl.a_shape[a] for a in self.a_off], [self.wl.b_shape[b] for b in self.b_off])

    def output(self, s):
        """Device view of problem s's C (whole, column-major m x n)."""
        it = self.wl.items[s]
        return self.C[self.c_off[s]:self.c_off[s] + it.m * it.n]


def path_id(g2, name: str) -> int:
    return {v: k for k, v in g2.PATH_NAMES.items()}[name]
