// shard.cpp -- ggemm_shard_group (include/ggemm_ext.h): partition of a group over devices.
//
// Problems are independent and their outputs disjoint, so a multi-GPU call needs no collective:
// every device runs its own handle on its own shard.  Balance comes from a cost estimate per
// problem (the planner's emulation model on a B200 device model, with the moduli count the
// adaptive rule would pick), longest-processing-time-first assignment, and two refinements:
//   * problems that share an A or B operand (same pointer, leading dimension, shape) form one
//     unit, so the operand's residues are computed once, on one device;
//   * a lone problem costing more than a shard's share is split into column blocks of 128
//     columns (B and C offsets), so a group smaller than the device count still spreads.
#include <algorithm>
#include <cmath>
#include <vector>

#include "ggemm_ext.h"
#include "internal.hpp"

namespace {

using g2::DeviceModel;

struct Unit {
  double cost;
  int src;        // original problem (column blocks) or -1 (component)
  int comp;       // component id for multi-problem units
  int j0, j1;     // column range for a single problem
};

int find(std::vector<int>& par, int x) {
  while (par[x] != x) {
    par[x] = par[par[x]];
    x = par[x];
  }
  return x;
}

// Modelled seconds of a problem restricted to `cols` columns: the planner's model of the
// emulated pipeline (adaptive moduli count), or native DGEMM when no count reaches 1e-15.
double problem_cost(const ggemm_problem_t& p, const DeviceModel& dm, int cols) {
  if (p.m <= 0 || cols <= 0) return 0.0;
  if (p.k <= 0 || p.alpha == 0.0) return 2.0 * p.m * cols * 8 / dm.recon_bw;  // C = beta C
  int N = g2::choose_num_moduli(p.k, 1e-15);
  if (N < 0) return g2::native_time(p.m, cols, p.k, p.beta != 0.0, dm);
  N = std::min(std::max(N, 2), g2::kMaxModuli);
  return g2::emu_time(p.m, cols, p.k, p.beta != 0.0, N, dm);
}

}  // namespace

extern "C" int ggemm_shard_group(const ggemm_problem_t* probs, int num, int S,
                                 ggemm_problem_t* out, int* out_shard, int* out_src, int out_cap,
                                 int* num_out) {
  if (num < 0 || S < 1 || (num > 0 && !probs) || !num_out || (out_cap > 0 && (!out || !out_shard || !out_src)))
    return GGEMM_ERR_INVALID;
  *num_out = 0;
  DeviceModel dm{};
  g2::device_model_init(&dm, 148);
  // components of problems linked through a shared A or B operand
  std::vector<int> par(num);
  for (int g = 0; g < num; ++g) par[g] = g;
  {
    std::vector<int> order(num);
    for (int g = 0; g < num; ++g) order[g] = g;
    auto link_by = [&](auto key_less, auto key_eq) {
      std::sort(order.begin(), order.end(), key_less);
      for (int i = 1; i < num; ++i)
        if (key_eq(order[i - 1], order[i])) {
          int a = find(par, order[i - 1]), b = find(par, order[i]);
          if (a != b) par[std::max(a, b)] = std::min(a, b);
        }
    };
    auto nonempty = [&](int g) { return probs[g].m > 0 && probs[g].n > 0 && probs[g].k > 0; };
    link_by(
        [&](int x, int y) {
          const auto &a = probs[x], &b = probs[y];
          if (a.A != b.A) return a.A < b.A;
          if (a.lda != b.lda) return a.lda < b.lda;
          if (a.m != b.m) return a.m < b.m;
          if (a.k != b.k) return a.k < b.k;
          return x < y;
        },
        [&](int x, int y) {
          const auto &a = probs[x], &b = probs[y];
          return nonempty(x) && nonempty(y) && a.A == b.A && a.lda == b.lda && a.m == b.m &&
                 a.k == b.k;
        });
    link_by(
        [&](int x, int y) {
          const auto &a = probs[x], &b = probs[y];
          if (a.B != b.B) return a.B < b.B;
          if (a.ldb != b.ldb) return a.ldb < b.ldb;
          if (a.n != b.n) return a.n < b.n;
          if (a.k != b.k) return a.k < b.k;
          return x < y;
        },
        [&](int x, int y) {
          const auto &a = probs[x], &b = probs[y];
          return nonempty(x) && nonempty(y) && a.B == b.B && a.ldb == b.ldb && a.n == b.n &&
                 a.k == b.k;
        });
  }
  std::vector<double> ccost(num, 0.0);
  std::vector<int> csize(num, 0);
  double total = 0.0;
  for (int g = 0; g < num; ++g) {
    const double c = problem_cost(probs[g], dm, probs[g].n);
    const int r = find(par, g);
    ccost[r] += c;
    csize[r] += 1;
    total += c;
  }
  const double target = total / S;
  std::vector<Unit> units;
  units.reserve((size_t)num + 64);
  for (int g = 0; g < num; ++g) {
    if (find(par, g) != g) continue;
    if (csize[g] == 1) {
      const ggemm_problem_t& p = probs[g];
      const int blocks_max = (p.n + 127) / 128;
      int blocks = 1;
      if (S > 1 && ccost[g] > target && blocks_max > 1)
        blocks = std::min(blocks_max, (int)std::ceil(ccost[g] / target - 1e-9));
      if (blocks <= 1) {
        units.push_back({ccost[g], g, -1, 0, p.n});
      } else {
        const int per = (blocks_max + blocks - 1) / blocks;  // 128-column blocks per unit
        for (int b = 0; b < blocks_max; b += per) {
          const int j0 = b * 128, j1 = std::min(p.n, (b + per) * 128);
          units.push_back({problem_cost(p, dm, j1 - j0), g, -1, j0, j1});
        }
      }
    } else {
      units.push_back({ccost[g], -1, g, 0, 0});
    }
  }
  std::stable_sort(units.begin(), units.end(),
                   [](const Unit& a, const Unit& b) { return a.cost > b.cost; });
  std::vector<double> load(S, 0.0);
  std::vector<int> unit_shard(units.size());
  for (size_t u = 0; u < units.size(); ++u) {
    int best = 0;
    for (int s = 1; s < S; ++s)
      if (load[s] < load[best]) best = s;
    load[best] += units[u].cost;
    unit_shard[u] = best;
  }
  // emit sub-problems shard by shard, in original problem order
  std::vector<int> shard_of_comp(num, -1);
  std::vector<std::vector<std::pair<int, int>>> blocks_of(num);  // (unit, shard) per problem
  for (size_t u = 0; u < units.size(); ++u) {
    if (units[u].src >= 0) blocks_of[units[u].src].push_back({(int)u, unit_shard[u]});
    else shard_of_comp[units[u].comp] = unit_shard[u];
  }
  int w = 0;
  for (int s = 0; s < S; ++s)
    for (int g = 0; g < num; ++g) {
      const ggemm_problem_t& p = probs[g];
      if (blocks_of[g].empty()) {
        if (shard_of_comp[find(par, g)] != s) continue;
        if (w >= out_cap) return GGEMM_ERR_WORKSPACE;
        out[w] = p;
        out_shard[w] = s;
        out_src[w] = g;
        ++w;
        continue;
      }
      std::vector<std::pair<int, int>> bl = blocks_of[g];
      std::sort(bl.begin(), bl.end(), [&](const std::pair<int, int>& a, const std::pair<int, int>& b) {
        return units[a.first].j0 < units[b.first].j0;
      });
      for (const auto& ub : bl) {
        if (ub.second != s) continue;
        const Unit& un = units[ub.first];
        if (w >= out_cap) return GGEMM_ERR_WORKSPACE;
        ggemm_problem_t q = p;
        q.n = un.j1 - un.j0;
        if (q.B) q.B = p.B + (size_t)un.j0 * p.ldb;
        if (q.C) q.C = p.C + (size_t)un.j0 * p.ldc;
        out[w] = q;
        out_shard[w] = s;
        out_src[w] = g;
        ++w;
      }
    }
  *num_out = w;
  return GGEMM_OK;
}
