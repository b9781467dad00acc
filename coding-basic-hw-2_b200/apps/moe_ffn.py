#!/usr/bin/env python
"""moe_ffn.py -- an FP64 Mixture-of-Experts FFN forward whose GEMMs all go through this
library's ggemm_grouped_dgemm (the reference's application caller bench/app/moe_ffn_fp64.cu, same
scenario: per-element fitting networks of machine-learned interatomic potentials, or MoE
surrogates inside FP64 solvers, where expert loads are data-dependent and skewed).

Pipeline (T tokens, d = d_model, f = d_ff, E experts, top-k):
  route    per token, k distinct experts from a Zipf(s) law over E (fixed seed) with gate weights
           summing to 1; tokens are grouped by expert (stable, deterministic);
  gather   Xg_e (m_e x d) <- the rows of X routed to expert e;
  up       grouped GEMM  H_e = Xg_e W1_e         (m_e x f)   [ggemm_grouped_dgemm]
  act      Ha = tanh(H);
  down     grouped GEMM  Yd_e = Ha_e W2_e         (m_e x d)   [ggemm_grouped_dgemm]
  scatter  Y[t] = sum_j g_tj Yd_{e_tj}[slot_tj]   (fixed order j: deterministic).
Matrices are column-major for the library: a row-major torch tensor of shape (r, c) is the
column-major c x r matrix, so H_e^T = W1_e^T Xg_e^T is computed as the column-major product
(f x d)(d x m_e) with the torch buffers as they are.

Correctness (as the reference app): against the same pipeline on NATIVE_LOOP (cuBLAS per
expert), err_cw = max |Y - Y_ref| / den with den the layer's first-order componentwise
sensitivity, reported over 2 gamma_n (<= 1: FP64 level).

  python coding-basic-hw-2_b200/apps/moe_ffn.py [--tokens 4096] [--experts 16] [--topk 2]
      [--d-model 1024] [--d-ff 2048] [--zipf 1.0] [--phi 0.5] [--reps 10]
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys

PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def load_pkg():
    if "ggemm_b200" in sys.modules:
        return sys.modules["ggemm_b200"]
    spec = importlib.util.spec_from_file_location("ggemm_b200", os.path.join(PKG, "__init__.py"),
                                                  submodule_search_locations=[PKG])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["ggemm_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def phi_fill(shape, phi, gen, device):
    import torch

    u = torch.rand(shape, generator=gen, device=device, dtype=torch.float64)
    z = torch.randn(shape, generator=gen, device=device, dtype=torch.float64)
    return (u - 0.5) * torch.exp(phi * z)


class MoELayer:
    """Weights of E experts and the routing of T tokens (deterministic for a seed)."""

    def __init__(self, tokens, experts, topk, d, f, zipf, phi, seed, device):
        import torch

        g = torch.Generator(device=device)
        g.manual_seed(seed)
        self.T, self.E, self.k, self.d, self.f = tokens, experts, topk, d, f
        self.X = phi_fill((tokens, d), phi, g, device)         # row-major T x d
        self.W1 = phi_fill((experts, d, f), phi, g, device)    # per expert row-major d x f
        self.W2 = phi_fill((experts, f, d), phi, g, device)
        # Zipf top-k routing: k distinct experts per token, sampled without replacement
        w = 1.0 / torch.arange(1, experts + 1, dtype=torch.float64, device=device) ** zipf
        choice = torch.multinomial(w.expand(tokens, experts), topk, replacement=False,
                                   generator=g)                 # T x k expert ids
        gate = torch.rand((tokens, topk), generator=g, device=device, dtype=torch.float64) + 0.1
        self.gate = gate / gate.sum(dim=1, keepdim=True)
        self.choice = choice
        flat = choice.reshape(-1)                                # token-major (t, j)
        order = torch.argsort(flat, stable=True)                # grouped by expert, stable
        self.order = order
        self.tok = order // topk                                 # token of each grouped row
        self.counts = torch.bincount(flat, minlength=experts).tolist()
        self.offsets = [0]
        for c in self.counts:
            self.offsets.append(self.offsets[-1] + c)


def forward(g2, layer, handle, path, cfg, bufs=None):
    """Y (T x d, row-major) of the layer; GEMMs through ggemm_grouped_dgemm on `path`."""
    import torch

    L = layer
    R = L.T * L.k
    if bufs is None:
        bufs = {"Xg": torch.empty((R, L.d), dtype=torch.float64, device=L.X.device),
                "H": torch.empty((R, L.f), dtype=torch.float64, device=L.X.device),
                "Yd": torch.empty((R, L.d), dtype=torch.float64, device=L.X.device)}
    Xg, H, Yd = bufs["Xg"], bufs["H"], bufs["Yd"]
    torch.index_select(L.X, 0, L.tok, out=Xg)                   # gather
    up, down = [], []
    for e in range(L.E):
        m, o = L.counts[e], L.offsets[e]
        if m == 0:
            continue
        # column-major: H_e^T (f x m) = W1_e^T (f x d) * Xg_e^T (d x m)
        up.append(dict(m=L.f, n=m, k=L.d, A=L.W1[e].data_ptr(), lda=L.f,
                       B=Xg.data_ptr() + 8 * o * L.d, ldb=L.d,
                       C=H.data_ptr() + 8 * o * L.f, ldc=L.f, alpha=1.0, beta=0.0))
        down.append(dict(m=L.d, n=m, k=L.f, A=L.W2[e].data_ptr(), lda=L.d,
                         B=H.data_ptr() + 8 * o * L.f, ldb=L.f,
                         C=Yd.data_ptr() + 8 * o * L.d, ldc=L.d, alpha=1.0, beta=0.0))
    P1, P2 = g2.make_problems(up), g2.make_problems(down)
    rc, _ = handle.grouped_dgemm(path, cfg, P1, len(up))
    if rc != 0:
        raise RuntimeError(f"up GEMM rc={rc}")
    torch.tanh(H, out=H)                                        # activation
    rc, _ = handle.grouped_dgemm(path, cfg, P2, len(down))
    if rc != 0:
        raise RuntimeError(f"down GEMM rc={rc}")
    # scatter: rows of Yd back to (token, slot) order, then the gated sum over slots j = 0..k-1
    Yslot = torch.empty_like(Yd)
    Yslot[L.order] = Yd
    Yslot = Yslot.view(L.T, L.k, L.d)
    Y = Yslot[:, 0, :] * L.gate[:, 0:1]
    for j in range(1, L.k):
        Y = Y + Yslot[:, j, :] * L.gate[:, j:j + 1]
    return Y, H  # H holds tanh(H) (activated in place)


def error_over_bound(layer, Y, Y_ref, Ha_ref):
    """max |Y - Y_ref| / den over 2 gamma_n: den = sum_j g_tj (|W2|^T (|tanh H| + |Xg||W1|)),
    n = max(d, f) + k + 4 (the reference app's diagnostic, bench/app/moe_ffn_fp64.cu).  Ha_ref:
    the activated hidden rows of the reference run (forward returns H after the tanh)."""
    import torch

    L = layer
    Xg = L.X[L.tok]
    absH = torch.empty_like(Ha_ref)
    for e in range(L.E):
        o, m = L.offsets[e], L.counts[e]
        if m:
            absH[o:o + m] = Ha_ref[o:o + m].abs() + Xg[o:o + m].abs() @ L.W1[e].abs()
    dn = torch.empty((L.T * L.k, L.d), dtype=torch.float64, device=Y.device)
    for e in range(L.E):
        o, m = L.offsets[e], L.counts[e]
        if m:
            dn[o:o + m] = absH[o:o + m] @ L.W2[e].abs()
    slot = torch.empty_like(dn)
    slot[L.order] = dn
    den = (slot.view(L.T, L.k, L.d) * L.gate.abs().unsqueeze(2)).sum(dim=1)
    n = max(L.d, L.f) + L.k + 4
    u = 2.0 ** -53
    gamma = n * u / (1 - n * u)
    err = ((Y - Y_ref).abs() / den.clamp_min(1e-300)).max().item()
    return err / (2 * gamma)


def main():
    import torch

    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--experts", type=int, default=16)
    ap.add_argument("--topk", type=int, default=2)
    ap.add_argument("--d-model", type=int, default=1024)
    ap.add_argument("--d-ff", type=int, default=2048)
    ap.add_argument("--zipf", type=float, default=1.0)
    ap.add_argument("--phi", type=float, default=0.5)
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--reps", type=int, default=10)
    args = ap.parse_args()
    g2 = load_pkg()
    dev = torch.device("cuda", 0)
    L = MoELayer(args.tokens, args.experts, args.topk, args.d_model, args.d_ff, args.zipf,
                 args.phi, args.seed, dev)
    R = L.T * L.k
    cfg = g2.config(0, 1e-15, 1, 0)
    s = torch.cuda.current_stream()
    with g2.Handle(args.experts, R * max(L.d, L.f) + L.E * L.d * L.f, R * max(L.d, L.f) * 2,
                   R * max(L.d, L.f), stream=s.cuda_stream) as h:
        bufs = {"Xg": torch.empty((R, L.d), dtype=torch.float64, device=dev),
                "H": torch.empty((R, L.f), dtype=torch.float64, device=dev),
                "Yd": torch.empty((R, L.d), dtype=torch.float64, device=dev)}
        Y_ref, H_ref = forward(g2, L, h, g2.PATH_NATIVE_LOOP, cfg)  # own buffers: kept
        out = {"tokens": L.T, "experts": L.E, "topk": L.k, "d_model": L.d, "d_ff": L.f,
               "expert_rows": L.counts}
        for name in ("native_grouped", "emu_grouped", "auto"):
            path = {v: k for k, v in g2.PATH_NAMES.items()}[name]
            for _ in range(2):
                Y, _ = forward(g2, L, h, path, cfg, bufs)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for _ in range(args.reps):
                Y, _ = forward(g2, L, h, path, cfg, bufs)
            e1.record(s)
            e1.synchronize()
            ms = e0.elapsed_time(e1) / args.reps
            flops = 2.0 * 2 * R * L.d * L.f
            out[name] = {"ms": ms, "gemm_tflops_effective": flops / ms / 1e9,
                         "err_over_bound": error_over_bound(L, Y, Y_ref, H_ref)}
    print(json.dumps(out))


if __name__ == "__main__":
    main()
